// W8A16 skinny GEMM kernels (see w8_gemm.cuh for the layout and modes),
// the one-time weight repack, and the reference-exact int8 quantiser.
#include <cooperative_groups.h>

#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace dfl {

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

// lane holds channels 4*lane .. 4*lane+3 of one 128-wide head; rotate
// (split-half neox: pairs d and d+64 live in lanes l and l^16).
__device__ __forceinline__ void rope_lane(float (&y)[4], int lane,
                                          const float2* __restrict__ cs_row) {
  float z[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) z[e] = __shfl_xor_sync(0xffffffffu, y[e], 16);
  const bool lo = lane < 16;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int i = (lane & 15) * 4 + e;  // frequency index 0..63
    const float2 t = __ldg(cs_row + i);
    const float c = t.x, s = t.y;
    // lo lane: x1 = y, x2 = z -> x1*cos - x2*sin ; hi lane: x1 = z, x2 = y -> x1*sin + x2*cos
    y[e] = lo ? (y[e] * c - z[e] * s) : (z[e] * s + y[e] * c);
  }
}

template <int MT, int MODE>
__global__ void __launch_bounds__(W8_WARPS * 32, (MT >= 8 ? 2 : 3)) w8_gemm_kernel(const W8Params p) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int MP = MT * 8;
  const int S = p.splits;
  const int tile = blockIdx.x / S;
  const int split = blockIdx.x % S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int nkb_all = p.K / 64;
  const int kb0 = split * nkb_all / S;
  const int nkb = (split + 1) * nkb_all / S - kb0;
  const int kslice = nkb * 64;
  const int nchunks = (kslice + W8_CHK - 1) / W8_CHK;
  __half* ring = reinterpret_cast<__half*>(smem);

  // 1) start streaming this warp's weights before touching activations
  const uint8_t* wp = p.w + w8_packed_offset(tile, kb0, warp, 0, 0, lane, p.K);
  constexpr size_t KB_STRIDE = (size_t)W8_WARPS * 2048;  // bytes between consecutive k64 blocks
  uint4 wb[W8_PD][4];
#pragma unroll
  for (int j = 0; j < W8_PD; ++j)
    if (j < nkb)
#pragma unroll
      for (int r = 0; r < 4; ++r) wb[j][r] = ldg_stream(wp + j * KB_STRIDE + r * 512);

  // 2) activation ring: chunk q holds X[0..MP)[kb0*64 + q*CHK, +CHK)
  auto load_chunk = [&](int q) {
    if (q < nchunks) {
      __half* st = ring + (size_t)(q % W8_NST) * MP * W8_XLD;
      const int k0 = q * W8_CHK;
      const int cpr = min(W8_CHK, kslice - k0) / 8;
      for (int idx = threadIdx.x; idx < MP * cpr; idx += W8_WARPS * 32) {
        const int m = idx / cpr, kk = (idx - m * cpr) * 8;
        const bool ok = m < p.M;
        const __half* src = p.x + (size_t)(ok ? m : 0) * p.K + (size_t)kb0 * 64 + k0 + kk;
        cp_async16_zfill(smem_u32(st + m * W8_XLD + kk), src, ok);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int q = 0; q < W8_NST - 1; ++q) load_chunk(q);

  float acc[2][MT][4];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[r][t][e] = 0.f;

  // 3) main loop over k64 blocks; a new ring chunk starts every CHK/64 blocks
  //    (the condition is uniform across the CTA, so the barrier is too)
  constexpr int KB_PER_CHUNK = W8_CHK / 64;
  const uint32_t ring_base = smem_u32(ring) + (uint32_t)((g * W8_XLD + c * 16) * 2);
  for (int kb = 0; kb < nkb; kb += W8_PD) {
#pragma unroll
    for (int j = 0; j < W8_PD; ++j) {
      const int k = kb + j;
      if (k < nkb) {
        if (k % KB_PER_CHUNK == 0) {
          cp_async_wait<W8_NST - 2>();
          __syncthreads();
          load_chunk(k / KB_PER_CHUNK + W8_NST - 1);
        }
        const uint4 cur0 = wb[j][0], cur1 = wb[j][1], cur2 = wb[j][2], cur3 = wb[j][3];
        if (k + W8_PD < nkb)
#pragma unroll
          for (int r = 0; r < 4; ++r) wb[j][r] = ldg_stream(wp + (size_t)(k + W8_PD) * KB_STRIDE + r * 512);
        const uint32_t kaddr = ring_base +
            (uint32_t)((((k / KB_PER_CHUNK) % W8_NST) * MP * W8_XLD + (k % KB_PER_CHUNK) * 64) * 2);
#pragma unroll
        for (int ih = 0; ih < 2; ++ih) {
          // activation row t*8+g, k = 16c + 8ih .. +7 : halves for MMAs i = 2ih, 2ih+1
          uint4 xq[MT];
#pragma unroll
          for (int t = 0; t < MT; ++t) xq[t] = lds128(kaddr + (uint32_t)(t * 8 * W8_XLD * 2 + ih * 16));
#pragma unroll
          for (int i = 2 * ih; i < 2 * ih + 2; ++i) {
            const uint32_t r0a0 = u8x2_to_f16x2(word_of(cur0, i), 0x5140);
            const uint32_t r0a2 = u8x2_to_f16x2(word_of(cur0, i), 0x5342);
            const uint32_t r0a1 = u8x2_to_f16x2(word_of(cur1, i), 0x5140);
            const uint32_t r0a3 = u8x2_to_f16x2(word_of(cur1, i), 0x5342);
            const uint32_t r1a0 = u8x2_to_f16x2(word_of(cur2, i), 0x5140);
            const uint32_t r1a2 = u8x2_to_f16x2(word_of(cur2, i), 0x5342);
            const uint32_t r1a1 = u8x2_to_f16x2(word_of(cur3, i), 0x5140);
            const uint32_t r1a3 = u8x2_to_f16x2(word_of(cur3, i), 0x5342);
#pragma unroll
            for (int t = 0; t < MT; ++t) {
              const uint32_t b0 = (i & 1) ? xq[t].z : xq[t].x;
              const uint32_t b1 = (i & 1) ? xq[t].w : xq[t].y;
              mma_f16_16816(acc[0][t], r0a0, r0a1, r0a2, r0a3, b0, b1);
              mma_f16_16816(acc[1][t], r1a0, r1a1, r1a2, r1a3, b0, b1);
            }
          }
        }
      }
    }
  }
  cp_async_wait<0>();

  // 4) partial tile -> shared (aliases the ring)
  constexpr int RS = MP + 1;
  float* red = reinterpret_cast<float*>(smem);
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int ch = warp * 32 + r * 16 + g;
      const int m = t * 8 + 2 * c;
      red[ch * RS + m] = acc[r][t][0];
      red[ch * RS + m + 1] = acc[r][t][1];
      red[(ch + 8) * RS + m] = acc[r][t][2];
      red[(ch + 8) * RS + m + 1] = acc[r][t][3];
    }
  cg::cluster_group cluster = cg::this_cluster();
  if (S > 1) cluster.sync(); else __syncthreads();

  // 5) epilogue: one item per activation row (the whole 128-channel tile); a
  //    warp owns an item; rank r of the cluster takes rows r, r+S, ...; the S
  //    partials are summed in rank order.
  constexpr int EPC = (MODE == kSiluMul) ? 2 : 4;  // outputs per lane
  for (int m = split + S * warp; m < p.M; m += S * W8_WARPS) {
    float v[4], u[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) { v[e] = 0.f; u[e] = 0.f; }
    const int ch0 = lane * EPC;
    for (int s = 0; s < S; ++s) {
      const float* rr = (S > 1) ? cluster.map_shared_rank(red, s) : red;
#pragma unroll
      for (int e = 0; e < EPC; ++e) {
        v[e] += rr[(ch0 + e) * RS + m];
        if (MODE == kSiluMul) u[e] += rr[(ch0 + 64 + e) * RS + m];
      }
    }
    const int gch = tile * W8_NT + ch0;  // global output channel of v[0]
#pragma unroll
    for (int e = 0; e < EPC; ++e) v[e] *= __ldg(p.scale + gch + e);

    if (MODE == kStore) {
      uint2 o;
      o.x = pack_f16x2(v[0], v[1]);
      o.y = pack_f16x2(v[2], v[3]);
      *reinterpret_cast<uint2*>(p.y + (size_t)m * p.N + gch) = o;
    } else if (MODE == kResid) {
      float4* hp = reinterpret_cast<float4*>(p.h_out + (size_t)m * p.N + gch);
      float4 hv = *hp;
      hv.x += v[0]; hv.y += v[1]; hv.z += v[2]; hv.w += v[3];
      *hp = hv;
      float ss = hv.x * hv.x + hv.y * hv.y + hv.z * hv.z + hv.w * hv.w;
      ss = warp_sum(ss);
      if (lane == 0) p.hstat_out[(size_t)tile * p.M + m] = ss;
    } else if (MODE == kSiluMul) {
      float o[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float gv = v[e];
        const float uv = u[e] * __ldg(p.scale + gch + 64 + e);
        o[e] = (gv / (1.0f + expf(-gv))) * uv;
      }
      *reinterpret_cast<uint32_t*>(p.act + (size_t)m * (p.N / 2) + tile * 64 + lane * 2) =
          pack_f16x2(o[0], o[1]);
    } else {  // kQKV: the tile is one head
      const int head = tile;
      const int bi = m / p.block, j = m - bi * p.block;
      const bool is_q = head < p.n_q_heads;
      const bool is_k = !is_q && head < p.n_q_heads + p.n_kv_heads;
      if (is_q || is_k) {
        const float* nw = is_q ? p.q_norm : p.k_norm;
        float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
        ss = warp_sum(ss);
        const float r = rsqrtf(ss / 128.0f + p.eps);
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = v[e] * r * __ldg(nw + lane * 4 + e);
        rope_lane(v, lane, p.rope + (size_t)(p.kv_row0 + j) * 64);
      }
      uint2 o;
      o.x = pack_f16x2(v[0], v[1]);
      o.y = pack_f16x2(v[2], v[3]);
      __half* dst;
      if (is_q) {
        dst = p.q_out + (((size_t)bi * p.n_q_heads + head) * p.block + j) * 128;
      } else {
        const int kvh = is_k ? head - p.n_q_heads : head - p.n_q_heads - p.n_kv_heads;
        __half* base = is_k ? p.k_out : p.v_out;
        dst = base + (((size_t)bi * p.n_kv_heads + kvh) * p.kv_rows + p.kv_row0 + j) * 128;
      }
      *reinterpret_cast<uint2*>(dst + lane * 4) = o;
    }
  }
  // keep this CTA's shared memory alive until every rank finished reading it
  if (S > 1) cluster.sync();
}

// ------------------------------------------------------------------ RMSNorm rows
// x[m, k] = f16(h[m, k] * rsqrt(sum_p hstat[p, m] / K + eps) * w[k]); one CTA per row
__global__ void rmsnorm_f16_kernel(const float* __restrict__ h, const float* __restrict__ hstat,
                                   int hparts, int M, int K, const float* __restrict__ w, float eps,
                                   __half* __restrict__ x) {
  const int m = blockIdx.x;
  __shared__ float part[32];
  float ss = 0.f;
  for (int q = threadIdx.x; q < hparts; q += blockDim.x) ss += hstat[(size_t)q * M + m];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) part[0] = rsqrtf(t / static_cast<float>(K) + eps);
  }
  __syncthreads();
  const float r = part[0];
  for (int k = threadIdx.x * 8; k < K; k += blockDim.x * 8) {
    const float4 a = *reinterpret_cast<const float4*>(h + (size_t)m * K + k);
    const float4 b = *reinterpret_cast<const float4*>(h + (size_t)m * K + k + 4);
    const float4 wa = *reinterpret_cast<const float4*>(w + k);
    const float4 wb = *reinterpret_cast<const float4*>(w + k + 4);
    uint4 o;
    o.x = pack_f16x2(a.x * r * wa.x, a.y * r * wa.y);
    o.y = pack_f16x2(a.z * r * wa.z, a.w * r * wa.w);
    o.z = pack_f16x2(b.x * r * wb.x, b.y * r * wb.y);
    o.w = pack_f16x2(b.z * r * wb.z, b.w * r * wb.w);
    *reinterpret_cast<uint4*>(x + (size_t)m * K + k) = o;
  }
}

// ------------------------------------------------------------------ repack
// Source channel r lands on output channel d = (r / grp) * gstride + r % grp + base
// (plain copy: grp >= n_src; gate/up interleave: grp 64, gstride 128, base 0 / 64).
__device__ __forceinline__ int w8_dst_channel(int r, int grp, int gstride, int base) {
  return (r / grp) * gstride + r % grp + base;
}

__global__ void w8_repack_kernel(const int8_t* __restrict__ src, int n_src, int K,
                                 uint8_t* __restrict__ dst, int grp, int gstride, int base) {
  const int nkb = K / 64;
  const size_t total = (size_t)n_src * nkb * 4;  // 16-byte pieces
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int c = idx & 3;
    const size_t rest = idx >> 2;
    const int kb = rest % nkb;
    const int r = rest / nkb;
    uint4 v = *reinterpret_cast<const uint4*>(src + (size_t)r * K + kb * 64 + 16 * c);
    v.x ^= 0x80808080u; v.y ^= 0x80808080u; v.z ^= 0x80808080u; v.w ^= 0x80808080u;
    const int d = w8_dst_channel(r, grp, gstride, base);
    const int tile = d / W8_NT, in_tile = d % W8_NT;
    const int warp = in_tile / 32, rb = (in_tile % 32) / 16, within = in_tile % 16;
    const int lane = 4 * (within % 8) + c, half = within / 8;
    *reinterpret_cast<uint4*>(dst + w8_packed_offset(tile, kb, warp, rb, half, lane, K)) = v;
  }
}

__global__ void w8_scale_kernel(const __half* __restrict__ s, int n_src, float* __restrict__ dst,
                                int grp, int gstride, int base) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n_src) return;
  dst[w8_dst_channel(r, grp, gstride, base)] = __half2float(s[r]);
}

// ------------------------------------------------------------------ quantiser
// ane_model.py:265-279: s = max|w|/127 (zero row -> 1/127), q = clip(rne(w/s))
__global__ void quantize_q8_kernel(const float* __restrict__ w, int ic, int8_t* __restrict__ q,
                                   __half* __restrict__ s) {
  const int row = blockIdx.x;
  const float* wr = w + (size_t)row * ic;
  float mx = 0.f;
  for (int k = threadIdx.x; k < ic; k += blockDim.x) mx = fmaxf(mx, fabsf(wr[k]));
  __shared__ float red[32];
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  float maxv = red[0];
  if (maxv == 0.f) maxv = 1.0f;
  const float sc = __fdiv_rn(maxv, 127.0f);
  for (int k = threadIdx.x; k < ic; k += blockDim.x) {
    float t = rintf(__fdiv_rn(wr[k], sc));
    t = fminf(fmaxf(t, -127.f), 127.f);
    q[(size_t)row * ic + k] = static_cast<int8_t>(t);
  }
  if (threadIdx.x == 0) s[row] = __float2half_rn(sc);
}

// ------------------------------------------------------------------ host
template <int MT, int MODE>
static cudaError_t launch_mt(const W8Params& p, size_t smem, cudaStream_t st) {
  auto kern = w8_gemm_kernel<MT, MODE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.N / W8_NT) * p.splits);
  cfg.blockDim = dim3(W8_WARPS * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int MODE>
static cudaError_t launch_mode(const W8Params& p, size_t smem, cudaStream_t st) {
  if (p.M <= 8) return launch_mt<1, MODE>(p, smem, st);
  if (p.M <= 16) return launch_mt<2, MODE>(p, smem, st);
  if (p.M <= 32) return launch_mt<4, MODE>(p, smem, st);
  return launch_mt<8, MODE>(p, smem, st);
}

// K-split (= cluster size, power of two, <= 8): the largest split whose grid
// still fits in one wave of three CTAs per SM, keeping >= 2 k64 blocks per CTA.
int w8_pick_splits(int N, int K, int M, int num_sms, int max_splits) {
  const int tiles = N / W8_NT;
  const int nkb = K / 64;
  const int per_sm = M > 32 ? 2 : 3;
  int s = 1;
  while (s * 2 <= max_splits && nkb / (s * 2) >= 2 && tiles * s * 2 <= per_sm * num_sms) s *= 2;
  return s;
}

size_t w8_smem_bytes(const W8Params& p) {
  const int mp = p.M <= 8 ? 8 : (p.M <= 16 ? 16 : (p.M <= 32 ? 32 : 64));
  const size_t ring = (size_t)W8_NST * mp * W8_XLD * 2;
  const size_t red = (size_t)W8_NT * (mp + 1) * 4;
  return ring > red ? ring : red;
}

static cudaError_t w8_gemm_launch_once(const W8Params& p, int mode, cudaStream_t st) {
  const size_t smem = w8_smem_bytes(p);
  if (mode == kQKV) return launch_mode<kQKV>(p, smem, st);
  if (mode == kResid) return launch_mode<kResid>(p, smem, st);
  if (mode == kSiluMul) return launch_mode<kSiluMul>(p, smem, st);
  if (mode == kStore) return launch_mode<kStore>(p, smem, st);
  return cudaErrorInvalidValue;
}

cudaError_t w8_gemm_launch(const W8Params& p, int mode, cudaStream_t st) {
  if (p.M < 1 || p.M > 64 || p.N % W8_NT || p.K % 64 || p.splits < 1 || p.splits > 8 ||
      p.K / 64 < p.splits)
    return cudaErrorInvalidValue;
  // a cluster that cannot be scheduled at this footprint is retried with half the split
  W8Params q = p;
  for (;;) {
    cudaError_t e = w8_gemm_launch_once(q, mode, st);
    if (e == cudaSuccess || q.splits == 1 ||
        (e != cudaErrorInvalidClusterSize && e != cudaErrorLaunchOutOfResources))
      return e;
    (void)cudaGetLastError();
    q.splits /= 2;
  }
}

cudaError_t rmsnorm_f16_launch(const float* h, const float* hstat, int hparts, int M, int K,
                               const float* w, float eps, __half* x, cudaStream_t st) {
  if (K % 8 || M < 1) return cudaErrorInvalidValue;
  rmsnorm_f16_kernel<<<M, 256, 0, st>>>(h, hstat, hparts, M, K, w, eps, x);
  return cudaGetLastError();
}

cudaError_t w8_repack_launch(const int8_t* src, int n_src, int K, uint8_t* dst, int grp,
                             int gstride, int base, cudaStream_t st) {
  if (n_src % 16 || K % 64) return cudaErrorInvalidValue;
  w8_repack_kernel<<<1024, 256, 0, st>>>(src, n_src, K, dst, grp, gstride, base);
  return cudaGetLastError();
}

cudaError_t w8_scale_launch(const __half* s, int n_src, float* dst, int grp, int gstride,
                            int base, cudaStream_t st) {
  w8_scale_kernel<<<(n_src + 255) / 256, 256, 0, st>>>(s, n_src, dst, grp, gstride, base);
  return cudaGetLastError();
}

cudaError_t quantize_q8_launch(const float* w, int oc, int ic, int8_t* q, __half* s,
                               cudaStream_t st) {
  if (oc < 1 || ic < 1) return cudaErrorInvalidValue;
  quantize_q8_kernel<<<oc, 256, 0, st>>>(w, ic, q, s);
  return cudaGetLastError();
}

}  // namespace dfl
