// Non-causal GQA block attention of the DFlash draft (dflash.py:310-319).
//
// One CTA per (batch, kv head, KV split).  All G = NQ/NKV query heads that
// share the kv head are processed together (R = G * block query rows), so each
// K/V row is read from HBM once per CTA.  One warp per 16-row m-tile; K/V
// tiles of 64 rows are double-buffered in shared memory with cp.async; QK^T
// and PV run on mma.sync m16n8k16 (f16 in, fp32 accumulate) with an online
// base-2 softmax.  Each CTA writes an unnormalised partial (O, m, l) that a
// combine kernel merges across splits in a fixed order.
//
// With `normrope` set the kernel also applies the per-head RMSNorm and neox
// RoPE of dflash.py:291-305 to the raw Q and K rows as they land in shared
// memory (the attention-only configuration); in the draft forward both are
// already applied by the projection epilogues.
//
// In the draft forward K/V rows are read through the KvMap of kernels.cuh:
// each sequence attends to its own logical rows [0, n_att), wherever the
// cache ring holds them.
#include <algorithm>

#include "kernels.cuh"

namespace dfl {


constexpr int AT_TK = 64;          // kv rows per shared tile
constexpr int AT_LD = 128 + 8;     // halves per shared row (+16 B pad)
constexpr int kAttnCtaCost = 6;    // per-CTA cost of a split in kv tiles (setup, partial write)
constexpr int kAttnMaxWaveSplits = 8;  // largest split the wave model may pick

__device__ __forceinline__ void normrope_row(__half* row, const float* w, const float2* cs_row,
                                             float eps, int lane) {
  // lane owns d = 4*lane .. 4*lane+3
  uint2 raw = *reinterpret_cast<uint2*>(row + lane * 4);
  __half2 h0 = *reinterpret_cast<__half2*>(&raw.x), h1 = *reinterpret_cast<__half2*>(&raw.y);
  float y[4] = {__low2float(h0), __high2float(h0), __low2float(h1), __high2float(h1)};
  float ss = warp_sum(y[0] * y[0] + y[1] * y[1] + y[2] * y[2] + y[3] * y[3]);
  const float r = rsqrtf(ss / 128.0f + eps);
#pragma unroll
  for (int e = 0; e < 4; ++e) y[e] = y[e] * r * __ldg(w + lane * 4 + e);
  float z[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) z[e] = __shfl_xor_sync(0xffffffffu, y[e], 16);
  const bool lo = lane < 16;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int i = (lane & 15) * 4 + e;
    const float2 t = __ldg(cs_row + i);
    const float c = t.x, s = t.y;
    y[e] = lo ? (y[e] * c - z[e] * s) : (z[e] * s + y[e] * c);
  }
  raw.x = pack_f16x2(y[0], y[1]);
  raw.y = pack_f16x2(y[2], y[3]);
  *reinterpret_cast<uint2*>(row + lane * 4) = raw;
}

__global__ void __launch_bounds__(384) attn_partial_kernel(const AttnParams p) {
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ __align__(16) uint8_t smem[];
  const int split = blockIdx.x, kvh = blockIdx.y, bi = blockIdx.z;
  const int G = p.nq / p.nkv;
  const int R = G * p.block;
  const int nwarps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int RP = nwarps * 16;

  __half* qs = reinterpret_cast<__half*>(smem);
  __half* ks = qs + (size_t)RP * AT_LD;               // [2][TK][LD]
  __half* vs = ks + (size_t)2 * AT_TK * AT_LD;        // [2][TK][LD]

  // logical kv rows of this sequence; with a KvMap they sit at ring slots
  const bool mapped = p.kv.nseq > 0;
  const int kv_len = mapped ? p.kv.seq[bi].n_att : p.kv_len;
  const int rs = mapped ? p.kv.seq[bi].rs_post : 0;
  const int kv0 = split * p.chunk;
  const int kv1 = min(kv_len, kv0 + p.chunk);
  const int ntiles = kv1 > kv0 ? (kv1 - kv0 + AT_TK - 1) / AT_TK : 0;

  const __half* qg = p.q + ((size_t)bi * p.nq + (size_t)kvh * G) * p.block * 128;
  const int kseq = mapped ? p.kv.seq[bi].cseq : bi;   // K/V store sequence
  const __half* kg = p.k + ((size_t)kseq * p.nkv + kvh) * (size_t)p.kv_cap * 128;
  const __half* vg = p.v + ((size_t)kseq * p.nkv + kvh) * (size_t)p.kv_cap * 128;

  // Q tile (rows >= R zero)
  for (int idx = threadIdx.x; idx < RP * 16; idx += blockDim.x) {
    const int r = idx >> 4, cc = (idx & 15) * 8;
    cp_async16_zfill(smem_u32(qs + (size_t)r * AT_LD + cc), qg + (size_t)min(r, R - 1) * 128 + cc,
                     r < R);
  }
  auto load_kv = [&](int t, int buf) {
    const int base = kv0 + t * AT_TK;
    for (int idx = threadIdx.x; idx < AT_TK * 16; idx += blockDim.x) {
      const int r = idx >> 4, cc = (idx & 15) * 8;
      const int row = base + r;
      const bool ok = row < kv1;
      const int lrow = ok ? row : 0;  // a valid address even when nothing is read
      const size_t off = (size_t)(mapped ? kv_slot(p.kv, lrow, rs) : lrow) * 128 + cc;
      cp_async16_zfill(smem_u32(ks + ((size_t)buf * AT_TK + r) * AT_LD + cc), kg + off, ok);
      cp_async16_zfill(smem_u32(vs + ((size_t)buf * AT_TK + r) * AT_LD + cc), vg + off, ok);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  const uint32_t qs_addr = smem_u32(qs);
  const uint32_t ks_addr = smem_u32(ks);
  const uint32_t vs_addr = smem_u32(vs);

  for (int t = 0; t < ntiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < ntiles) load_kv(t + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (p.normrope) {
      if (t == 0) {
        for (int r = warp; r < R; r += nwarps)
          normrope_row(qs + (size_t)r * AT_LD, p.q_norm,
                       p.rope + (size_t)(p.q_row0 + r % p.block) * 64, p.eps, lane);
      }
      const int base = kv0 + t * AT_TK;
      for (int r = warp; r < AT_TK; r += nwarps)
        if (base + r < kv1)
          normrope_row(ks + ((size_t)buf * AT_TK + r) * AT_LD, p.k_norm,
                       p.rope + (size_t)(p.k_row0 + base + r) * 64, p.eps, lane);
      __syncthreads();
    }

    // S = Q K^T for this warp's 16 rows x 64 kv
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[i][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4(qs_addr + (uint32_t)(((warp * 16 + (lane & 15)) * AT_LD + kk * 16 + (lane >> 4) * 8) * 2),
                  a0, a1, a2, a3);
#pragma unroll
      for (int nt = 0; nt < 8; nt += 2) {
        const int mat = lane >> 3;
        const int krow = nt * 8 + (lane & 7) + (mat >> 1) * 8;
        const int kcol = kk * 16 + (mat & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(ks_addr + (uint32_t)((((size_t)buf * AT_TK + krow) * AT_LD + kcol) * 2), b0, b1,
                    b2, b3);
        mma_f16_16816(s[nt], a0, a1, a2, a3, b0, b1);
        mma_f16_16816(s[nt + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // scale, mask, online softmax (rows g and g+8 of the m-tile)
    const int base = kv0 + t * AT_TK;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = base + nt * 8 + 2 * c + (e & 1);
        float val = s[nt][e] * p.scale_log2;
        if (col >= kv1) val = -INFINITY;
        s[nt][e] = val;
        mx[e >> 1] = fmaxf(mx[e >> 1], val);
      }
    }
    float corr[2], msafe[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      const float mnew = fmaxf(m_run[h], mx[h]);
      msafe[h] = (mnew == -INFINITY) ? 0.f : mnew;
      corr[h] = exp2f(m_run[h] - msafe[h]);
      m_run[h] = mnew;
    }
    float ls[2] = {0.f, 0.f};
    uint32_t pa[8][2];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = exp2f(s[nt][0] - msafe[0]);
      const float p1 = exp2f(s[nt][1] - msafe[0]);
      const float p2 = exp2f(s[nt][2] - msafe[1]);
      const float p3 = exp2f(s[nt][3] - msafe[1]);
      ls[0] += p0 + p1;
      ls[1] += p2 + p3;
      pa[nt][0] = pack_f16x2(p0, p1);
      pa[nt][1] = pack_f16x2(p2, p3);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      ls[h] += __shfl_xor_sync(0xffffffffu, ls[h], 1);
      ls[h] += __shfl_xor_sync(0xffffffffu, ls[h], 2);
      l_run[h] = l_run[h] * corr[h] + ls[h];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= corr[0]; o[i][1] *= corr[0];
      o[i][2] *= corr[1]; o[i][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int kt = 0; kt < 4; ++kt) {
      const uint32_t a0 = pa[2 * kt][0], a1 = pa[2 * kt][1];
      const uint32_t a2 = pa[2 * kt + 1][0], a3 = pa[2 * kt + 1][1];
#pragma unroll
      for (int dt = 0; dt < 16; dt += 2) {
        const int mat = lane >> 3;
        const int vrow = kt * 16 + (lane & 7) + (mat & 1) * 8;
        const int vcol = dt * 8 + (mat >> 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(vs_addr + (uint32_t)((((size_t)buf * AT_TK + vrow) * AT_LD + vcol) * 2), b0,
                          b1, b2, b3);
        mma_f16_16816(o[dt], a0, a1, a2, a3, b0, b1);
        mma_f16_16816(o[dt + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // buffer `buf` is refilled by the next iteration's prefetch
  }

  // partials
  const size_t pbase = (((size_t)bi * p.nkv + kvh) * p.splits + split) * (size_t)R;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = warp * 16 + g + h * 8;
    if (r < R) {
      float* orow = p.opart + (pbase + r) * 128;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt)
        *reinterpret_cast<float2*>(orow + dt * 8 + 2 * c) = make_float2(o[dt][2 * h], o[dt][2 * h + 1]);
      if (c == 0) {
        p.mpart[pbase + r] = m_run[h];
        p.lpart[pbase + r] = l_run[h];
      }
    }
  }
}

// Merge of the split partials of one (sequence bi, head, block row j): one
// warp, lanes split the splits for the max / denominator and the head dims
// for the weighted sum.  Returns lane's 4 output dims as f16.  The maxima,
// the denominators and the first ROWS partial rows are all loaded before any
// is used, so up to ROWS splits cost one L2 round trip; the sums run in split
// order.  The fused limb merge takes ROWS = 20 (17 splits at the 27B draft's
// ctx 4096 step); the plain merge, launched with many CTAs per SM at large
// batch, keeps its registers low with 8.
template <int AT_MERGE_ROWS>
__device__ __forceinline__ uint2 attn_merge_row(const AttnParams& p, int bi, int head, int j, int lane) {
  const int G = p.nq / p.nkv;
  const int R = G * p.block;
  const int kvh = head / G;
  const int r = (head - kvh * G) * p.block + j;
  const size_t base = (((size_t)bi * p.nkv + kvh) * p.splits) * (size_t)R + r;
  auto orow = [&](int s) {
    return __ldcg(reinterpret_cast<const float4*>(p.opart + (base + (size_t)s * R) * 128 + lane * 4));
  };
  float mv0 = -INFINITY, lv0 = 0.f;
  if (lane < p.splits) {
    mv0 = p.mpart[base + (size_t)lane * R];
    lv0 = p.lpart[base + (size_t)lane * R];
  }
  float4 ov[AT_MERGE_ROWS];
#pragma unroll
  for (int t = 0; t < AT_MERGE_ROWS; ++t) ov[t] = t < p.splits ? orow(t) : make_float4(0.f, 0.f, 0.f, 0.f);
  float M = mv0;
  for (int s = lane + 32; s < p.splits; s += 32) M = fmaxf(M, p.mpart[base + (size_t)s * R]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  const float Ms = (M == -INFINITY) ? 0.f : M;
  float L = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s0 = 0; s0 < p.splits; s0 += 32) {
    const int s = s0 + lane;
    float w = 0.f;
    if (s < p.splits) {
      const size_t idx = base + (size_t)s * R;
      w = exp2f((s0 == 0 ? mv0 : p.mpart[idx]) - Ms);
      L += (s0 == 0 ? lv0 : p.lpart[idx]) * w;
    }
    const int n = min(32, p.splits - s0);
    for (int t0 = 0; t0 < n; t0 += AT_MERGE_ROWS) {
      if (s0 + t0 > 0) {
#pragma unroll
        for (int t = 0; t < AT_MERGE_ROWS; ++t)
          ov[t] = t0 + t < n ? orow(s0 + t0 + t) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int t = 0; t < AT_MERGE_ROWS; ++t) {
        const float wt = __shfl_sync(0xffffffffu, w, (t0 + t) & 31);
        if (t0 + t < n) {
          acc[0] += ov[t].x * wt; acc[1] += ov[t].y * wt; acc[2] += ov[t].z * wt; acc[3] += ov[t].w * wt;
        }
      }
    }
  }
  L = warp_sum(L);
  const float inv = 1.0f / L;
  uint2 pk;
  pk.x = pack_f16x2(acc[0] * inv, acc[1] * inv);
  pk.y = pack_f16x2(acc[2] * inv, acc[3] * inv);
  return pk;
}

// merge split partials -> out [b*B, NQ*128] f16 (row = bi*B + j, col = head*128 + d);
// one warp per (batch, head, block row)
__global__ void attn_combine_kernel(const AttnParams p, __half* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int bi = blockIdx.y;
  if (row >= p.nq * p.block) return;
  const int head = row / p.block, j = row % p.block;
  const uint2 pk = attn_merge_row<8>(p, bi, head, j, lane);
  *reinterpret_cast<uint2*>(out + ((size_t)bi * p.block + j) * ((size_t)p.nq * 128) +
                            (size_t)head * 128 + lane * 4) = pk;
  if (p.omax) {  // per (head, row) max |out| for the o-projection's limb split
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&pk.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&pk.y));
    const float mx = warp_max(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y))));
    if (lane == 0) p.omax[(size_t)head * gridDim.y * p.block + (size_t)bi * p.block + j] = mx;
  }
}

// The merge fused with the o-projection's limb split.  One cluster of
// C = ceil(NQ / 8) CTAs per activation row m = bi * B + j; CTA c merges heads
// 8c .. 8c + 7 (a warp each), and the cluster exchanges the maxima of the f16
// rows through distributed shared memory, so every CTA splits its own
// columns with the row's power-of-two scale.  The limbs and scales are those
// that attn_combine_kernel followed by the standalone limb split produce.
__global__ void __launch_bounds__(256, 2) attn_combine_limbs_kernel(const AttnParams p, int M, int MP,
                                                                 int8_t* __restrict__ xl,
                                                                 float* __restrict__ xscale) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float wmax[8];
  __shared__ float cmax;
  const int K = p.nq * 128;
  const int c = blockIdx.x, m = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = c * 8 + warp;
  const size_t col = (size_t)head * 128 + lane * 4;
  int8_t* o0 = xl + (size_t)m * K + col;
  int8_t* o1 = o0 + (size_t)MP * K;
  int8_t* o2 = o1 + (size_t)MP * K;
  if (m >= M) {  // padding rows: the whole cluster takes this branch
    if (head < p.nq) {
      *reinterpret_cast<uint32_t*>(o0) = 0u;
      *reinterpret_cast<uint32_t*>(o1) = 0u;
      *reinterpret_cast<uint32_t*>(o2) = 0u;
    }
    if (c == 0 && threadIdx.x == 0) xscale[m] = 1.f;
    return;
  }
  const int bi = m / p.block, j = m - bi * p.block;
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (head < p.nq) {
    const uint2 pk = attn_merge_row<20>(p, bi, head, j, lane);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&pk.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&pk.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  }
  const float mx = warp_max(fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3]))));
  if (lane == 0) wmax[warp] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t = fmaxf(t, wmax[w]);
    cmax = t;
  }
  cluster_arrive_release();
  cluster_wait_acquire();  // every CTA of the row has its maximum in place
  float rmx = 0.f;
  for (uint32_t r = 0; r < gridDim.x; ++r) rmx = fmaxf(rmx, ld_cluster_f32(&cmax, r));
  cluster_arrive_release();  // done reading the peers' shared memory
  int e;
  frexpf(rmx, &e);  // every |x| <= rmx < 2^e
  const float up = ldexpf(1.f, 20 - e);
  if (c == 0 && threadIdx.x == 0) xscale[m] = ldexpf(1.f, e - 20);
  if (head < p.nq) {
    int8_t l[3][4];
#pragma unroll
    for (int t = 0; t < 4; ++t) limbs_of(v[t], up, l[0][t], l[1][t], l[2][t]);
    *reinterpret_cast<char4*>(o0) = make_char4(l[0][0], l[0][1], l[0][2], l[0][3]);
    *reinterpret_cast<char4*>(o1) = make_char4(l[1][0], l[1][1], l[1][2], l[1][3]);
    *reinterpret_cast<char4*>(o2) = make_char4(l[2][0], l[2][1], l[2][2], l[2][3]);
  }
  cluster_wait_acquire();  // no CTA leaves while a peer may still read its maximum
}

size_t attn_smem_bytes(int nq, int nkv, int block) {
  const int R = nq / nkv * block;
  const int RP = (R + 15) / 16 * 16;
  return ((size_t)RP * AT_LD + (size_t)4 * AT_TK * AT_LD) * 2;
}

// Upper bound of attn_pick_split's count for any kv length (workspace sizing)
int attn_max_splits(int batch, int nkv, int num_sms, int rows) {
  const int per = batch * nkv;
  const int s = (num_sms + per - 1) / per;
  return rows > 128 ? std::max(s, kAttnMaxWaveSplits) : s;
}

// Choose the KV split.  With at most 128 query rows per kv head the split
// covers the SMs about once (b * NKV * splits >= SMs; grids of two CTAs per SM
// take the two-stage ring).  With more rows (two query groups) the tcgen05
// kernel runs one CTA per SM, and the split minimises
//   waves * (kv tiles per CTA + kAttnCtaCost),   waves = ceil(b * NKV * splits / SMs),
// so that no partial second wave doubles the time: at ctx 32768 and batch 1,
// 18 splits (144 CTAs) take 69 us where 19 (152 CTAs, 4 in a second wave) took
// 117 us; at batch 16, 8 splits (1024 CTAs, 6.9 waves) take 886 us against 964
// for 2.  kAttnCtaCost, the per-CTA setup and partial write in tile units,
// fits the c4 sweep (1, 2, 8, 15, 18, 37 and 55 splits at ctx 8K-32K); it was
// 4 until the tiles got faster, which left batch 16 / ctx 16K on 8 splits
// (342 us) where one split covers 128 SMs in one wave.
void attn_pick_split(int batch, int nkv, int kv_len, int num_sms, int rows, int* chunk, int* splits) {
  const int per = batch * nkv;
  const int tiles = (kv_len + AT_TK - 1) / AT_TK;
  int s = (num_sms + per - 1) / per;
  if (rows > 128) {
    const int cap = attn_max_splits(batch, nkv, num_sms, rows);
    long long best = -1;
    for (int c = 1; c <= cap && c <= tiles; ++c) {
      const int per_cta = (tiles + c - 1) / c;
      const int se = (tiles + per_cta - 1) / per_cta;
      const long long waves = ((long long)per * se + num_sms - 1) / num_sms;
      const long long cost = waves * (per_cta + kAttnCtaCost);
      if (best < 0 || cost < best) {
        best = cost;
        s = se;
      }
    }
  }
  if (s > tiles) s = tiles;
  if (s < 1) s = 1;
  int ch = (kv_len + s - 1) / s;
  ch = (ch + AT_TK - 1) / AT_TK * AT_TK;
  s = (kv_len + ch - 1) / ch;
  *chunk = ch;
  *splits = s;
}

cudaError_t attn_launch(const AttnParams& p, int batch, __half* out, cudaStream_t st) {
  const int G = p.nq / p.nkv;
  const int R = G * p.block;
  if (p.nq % p.nkv || R < 1 || R > 192 || p.kv_len < 1 || p.chunk % AT_TK) return cudaErrorInvalidValue;
  const int nwarps = (R + 15) / 16;
  const size_t smem = attn_smem_bytes(p.nq, p.nkv, p.block);
  cudaError_t e = cudaFuncSetAttribute(attn_partial_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  DFL_TRY(max_smem_carveout(attn_partial_kernel));
  e = launch_pdl(attn_partial_kernel, dim3(p.splits, p.nkv, batch), dim3(nwarps * 32), smem, st, p);
  if (e != cudaSuccess) return e;
  return attn_combine_launch(p, batch, out, st);
}

cudaError_t attn_combine_launch(const AttnParams& p, int batch, __half* out, cudaStream_t st) {
  const int rows = p.nq * p.block;
  DFL_TRY(max_smem_carveout(attn_combine_kernel));
  return launch_pdl(attn_combine_kernel, dim3((rows + 7) / 8, batch), dim3(256), 0, st, p, out);
}

cudaError_t attn_combine_limbs_launch(const AttnParams& p, int batch, const AttnLimbOut& lo, cudaStream_t st) {
  const int C = (p.nq + 7) / 8;
  if (C > 8 || lo.M != batch * p.block || lo.M < 1 || lo.M > 64 || !lo.xl || !lo.xscale)
    return cudaErrorInvalidValue;
  const int mp = (lo.M + 15) / 16 * 16;
  return launch_pdl_cluster(attn_combine_limbs_kernel, dim3(C, mp), dim3(256), (unsigned)C, st, p, lo.M, mp,
                            lo.xl, lo.xscale);
}

}  // namespace dfl
