// Soft anchor (mirror_sd/generate.py:1422-1436): position 0 of a draft block
// is embedded as the softmax-weighted sum of the top-k token embeddings under
// the previous verify step's logits at the correction position:
//   ids    = the k largest logits, larger first, lower index first on ties
//            (a stable argsort of -logits)
//   w      = softmax(logits[ids]) in fp32
//   anchor = bf16(sum_q w_q * E[ids_q])        (fp32 products, summed q = 0..k-1)
//
// One launch per step: grid (G, batch).  Each CTA scans a contiguous slice of
// its row's logits, every thread keeping a register-resident sorted top-LK
// list, and the CTA merges its threads' lists into the slice's top-k, written
// to the candidate workspace.  The last CTA of the row to arrive (a counter
// per row, reset by that CTA) merges the G * k candidates and forms the
// weighted embedding sum.  E is either row-major [V, H] or the 128-row
// swizzled vocabulary tiles the lm_head kernel streams (lm_pack_kernel), so
// the draft forward reads the one copy of the embedding it already holds.
#include <algorithm>

#include "kernels.cuh"

namespace dfl {

constexpr int SA_THREADS = 256;

// (value, index) order: larger value first, lower index on ties
__device__ __forceinline__ bool sa_better(float v, int i, float w, int j) {
  return v > w || (v == w && i < j);
}

template <int LK>
struct SaList {
  float v[LK];
  int i[LK];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int q = 0; q < LK; ++q) {
      v[q] = -INFINITY;
      i[q] = 0x7fffffff;
    }
  }
  // insert keeping the list sorted best-first; fully unrolled so the list
  // stays in registers
  __device__ __forceinline__ void push(float x, int idx) {
    if (!sa_better(x, idx, v[LK - 1], i[LK - 1])) return;
    v[LK - 1] = x;
    i[LK - 1] = idx;
#pragma unroll
    for (int q = LK - 1; q > 0; --q) {
      if (sa_better(v[q], i[q], v[q - 1], i[q - 1])) {
        const float tv = v[q];
        v[q] = v[q - 1];
        v[q - 1] = tv;
        const int ti = i[q];
        i[q] = i[q - 1];
        i[q - 1] = ti;
      }
    }
  }
};

template <int LK>
struct SaShared {
  float lv[SA_THREADS * LK];
  int li[SA_THREADS * LK];
  int head[SA_THREADS];
  float rv[SA_THREADS / 32];
  int ri[SA_THREADS / 32], rt[SA_THREADS / 32];
  float sel_v[LK];
  int sel_i[LK];
  int last;
};

// the CTA's top-k of its threads' lists -> sel_v / sel_i (k rounds of a
// block-wide arg-best over the lists' heads)
template <int LK>
__device__ void sa_merge(SaShared<LK>& s, const SaList<LK>& l, int k) {
  const int t = threadIdx.x;
#pragma unroll
  for (int q = 0; q < LK; ++q) {
    s.lv[t * LK + q] = l.v[q];
    s.li[t * LK + q] = l.i[q];
  }
  s.head[t] = 0;
  __syncthreads();
  for (int round = 0; round < k; ++round) {
    const int h = s.head[t];
    float bv = h < LK ? s.lv[t * LK + h] : -INFINITY;
    int bi = h < LK ? s.li[t * LK + h] : 0x7fffffff;
    int bt = t;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const int ot = __shfl_xor_sync(0xffffffffu, bt, o);
      if (sa_better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
        bt = ot;
      }
    }
    if ((t & 31) == 0) {
      s.rv[t >> 5] = bv;
      s.ri[t >> 5] = bi;
      s.rt[t >> 5] = bt;
    }
    __syncthreads();
    if (t == 0) {
      int best = 0;
      for (int w = 1; w < SA_THREADS / 32; ++w)
        if (sa_better(s.rv[w], s.ri[w], s.rv[best], s.ri[best])) best = w;
      s.sel_v[round] = s.rv[best];
      s.sel_i[round] = s.ri[best];
      s.head[s.rt[best]] += 1;
    }
    __syncthreads();
  }
}

// 16-byte chunk holding E[v, c .. c+7]
template <bool TILED>
__device__ __forceinline__ const uint4* sa_erow(const void* E, int H, int v, int c) {
  if (!TILED) return reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(E) + (size_t)v * H + c);
  const int nkb = H / 64, r = v & 127, j = (c & 63) >> 3;
  const size_t off = (((size_t)(v >> 7) * nkb + (c >> 6)) * 128 + r) * 128 + ((j ^ (r & 7)) << 4);
  return reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(E) + off);
}

template <int LK, bool TILED, bool BF16>
__global__ void __launch_bounds__(SA_THREADS) soft_anchor_kernel(const SaParams p) {
  __shared__ SaShared<LK> s;
  griddep_wait();
  griddep_launch_dependents();
  const int row = blockIdx.y, G = gridDim.x;
  const int per = (p.V + G - 1) / G;
  const int v0 = blockIdx.x * per, v1 = min(p.V, v0 + per);
  SaList<LK> l;
  l.init();
  if (BF16) {
    const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(p.logits) + (size_t)row * p.ld;
    for (int v = v0 + threadIdx.x; v < v1; v += SA_THREADS) l.push(__bfloat162float(x[v]), v);
  } else {
    const float* x = static_cast<const float*>(p.logits) + (size_t)row * p.ld;
    for (int v = v0 + threadIdx.x; v < v1; v += SA_THREADS) l.push(x[v], v);
  }
  sa_merge<LK>(s, l, p.k);
  float* cv = p.cand_v + ((size_t)row * G + blockIdx.x) * LK;
  int* ci = p.cand_i + ((size_t)row * G + blockIdx.x) * LK;
  if (threadIdx.x < p.k) {
    cv[threadIdx.x] = s.sel_v[threadIdx.x];
    ci[threadIdx.x] = s.sel_i[threadIdx.x];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s.last = atomicAdd(p.counter + row, 1) == G - 1;
  __syncthreads();
  if (!s.last) return;
  __threadfence();
  // last CTA of the row: top-k of the G * k candidates
  l.init();
  const float* av = p.cand_v + (size_t)row * G * LK;
  const int* ai = p.cand_i + (size_t)row * G * LK;
  for (int c = threadIdx.x; c < G * p.k; c += SA_THREADS) {
    const int g = c / p.k, q = c - g * p.k;
    l.push(__ldcg(av + g * LK + q), __ldcg(ai + g * LK + q));
  }
  __syncthreads();
  sa_merge<LK>(s, l, p.k);
  if (threadIdx.x == 0) p.counter[row] = 0;
  // softmax over the selected logits: the reference's weights, then the sum
  float w[LK];
  float den = 0.f;
  const float mx = s.sel_v[0];
#pragma unroll
  for (int q = 0; q < LK; ++q) {
    w[q] = q < p.k ? expf(s.sel_v[q] - mx) : 0.f;
    den = __fadd_rn(den, w[q]);
  }
#pragma unroll
  for (int q = 0; q < LK; ++q) w[q] = __fdiv_rn(w[q], den);
  __nv_bfloat16* out = p.out + (size_t)row * p.out_ld;
  for (int c = threadIdx.x * 8; c < p.H; c += SA_THREADS * 8) {
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    for (int q = 0; q < p.k; ++q) {
      const int id = s.sel_i[q];
      if (id < 0 || id >= p.V) continue;   // fewer than k orderable logits (NaN row)
      const uint4 raw = __ldg(sa_erow<TILED>(p.E, p.H, id, c));
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(b[e]);
        acc[2 * e] = __fadd_rn(acc[2 * e], __fmul_rn(w[q], f.x));
        acc[2 * e + 1] = __fadd_rn(acc[2 * e + 1], __fmul_rn(w[q], f.y));
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + c) = o;
  }
}

int soft_anchor_ctas(int V, int rows, int num_sms) {
  const int by_len = (V + 4 * SA_THREADS - 1) / (4 * SA_THREADS);
  const int by_sms = std::max(1, (2 * num_sms) / std::max(rows, 1));
  return std::max(1, std::min(std::min(by_len, by_sms), kSaMaxCtas));
}

template <int LK, bool TILED>
static cudaError_t sa_launch_t(const SaParams& p, int G, int rows, cudaStream_t st) {
  if (p.logits_bf16) {
    DFL_TRY(max_smem_carveout(soft_anchor_kernel<LK, TILED, true>));
    return launch_pdl(soft_anchor_kernel<LK, TILED, true>, dim3(G, rows), dim3(SA_THREADS), 0, st, p);
  }
  DFL_TRY(max_smem_carveout(soft_anchor_kernel<LK, TILED, false>));
  return launch_pdl(soft_anchor_kernel<LK, TILED, false>, dim3(G, rows), dim3(SA_THREADS), 0, st, p);
}

cudaError_t soft_anchor_launch(const SaParams& p, int rows, bool e_tiled, int num_sms, cudaStream_t st) {
  if (rows < 1 || p.V < 1 || p.H < 8 || p.H % 8 || p.k < 1 || p.k > kSaMaxK || p.k > p.V ||
      (e_tiled && p.H % 64))
    return cudaErrorInvalidValue;
  const int G = soft_anchor_ctas(p.V, rows, num_sms);
  if (p.k <= 8) return e_tiled ? sa_launch_t<8, true>(p, G, rows, st) : sa_launch_t<8, false>(p, G, rows, st);
  return e_tiled ? sa_launch_t<16, true>(p, G, rows, st) : sa_launch_t<16, false>(p, G, rows, st);
}

}  // namespace dfl
