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

template <int MT, int MODE, int XSRC>
__global__ void __launch_bounds__(W8_WARPS * 32) w8_gemm_kernel(const W8Params p) {
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
  const int xstride = kslice + 8;  // halves; +16 B per row keeps ldmatrix-style reads conflict free
  __half* xs = reinterpret_cast<__half*>(smem);
  float* rstd_s = reinterpret_cast<float*>(smem + (size_t)MP * xstride * 2);

  // 1) start streaming this warp's weights before touching activations
  const int rb0 = (tile * W8_NT + warp * 32) >> 4;
  const uint8_t* wp0 = p.w + w8_packed_offset(rb0, kb0, 0, lane, p.K);
  const uint8_t* wp1 = p.w + w8_packed_offset(rb0 + 1, kb0, 0, lane, p.K);
  uint4 wb[W8_PD][4];
#pragma unroll
  for (int j = 0; j < W8_PD; ++j) {
    if (j < nkb) {
      wb[j][0] = ldg_stream(wp0 + (size_t)j * 1024);
      wb[j][1] = ldg_stream(wp0 + (size_t)j * 1024 + 512);
      wb[j][2] = ldg_stream(wp1 + (size_t)j * 1024);
      wb[j][3] = ldg_stream(wp1 + (size_t)j * 1024 + 512);
    }
  }

  // 2) activations -> shared (f16), rows >= M are zero
  if (XSRC == kXHNorm) {
    if (threadIdx.x < MP) {
      const int m = threadIdx.x;
      float r = 0.f;
      if (m < p.M) {
        float ss = 0.f;
        for (int q = 0; q < p.hparts; ++q) ss += p.hstat[(size_t)q * p.M + m];
        r = rsqrtf(ss / static_cast<float>(p.K) + p.eps);
      }
      rstd_s[m] = r;
    }
    __syncthreads();
  }
  {
    const int cpr = kslice / 8;  // 16-byte chunks per row
    for (int idx = threadIdx.x; idx < MP * cpr; idx += blockDim.x) {
      const int m = idx / cpr;
      const int kk = (idx - m * cpr) * 8;
      uint4 val = make_uint4(0, 0, 0, 0);
      if (m < p.M) {
        const size_t gk = (size_t)kb0 * 64 + kk;
        if (XSRC == kXF16) {
          val = *reinterpret_cast<const uint4*>(p.x + (size_t)m * p.K + gk);
        } else {
          const float4 a = *reinterpret_cast<const float4*>(p.h + (size_t)m * p.K + gk);
          const float4 b = *reinterpret_cast<const float4*>(p.h + (size_t)m * p.K + gk + 4);
          const float4 wa = *reinterpret_cast<const float4*>(p.norm_w + gk);
          const float4 wb4 = *reinterpret_cast<const float4*>(p.norm_w + gk + 4);
          const float r = rstd_s[m];
          val.x = pack_f16x2(a.x * r * wa.x, a.y * r * wa.y);
          val.y = pack_f16x2(a.z * r * wa.z, a.w * r * wa.w);
          val.z = pack_f16x2(b.x * r * wb4.x, b.y * r * wb4.y);
          val.w = pack_f16x2(b.z * r * wb4.z, b.w * r * wb4.w);
        }
      }
      *reinterpret_cast<uint4*>(xs + (size_t)m * xstride + kk) = val;
    }
  }
  __syncthreads();

  // 3) main loop over this CTA's K slice, k64 blocks
  float acc[2][MT][4];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[r][t][e] = 0.f;

  const uint32_t xs_base = smem_u32(xs) + (uint32_t)((g * xstride + c * 16) * 2);
  for (int kbb = 0; kbb < nkb; kbb += W8_PD) {
#pragma unroll
    for (int j = 0; j < W8_PD; ++j) {
      const int kb = kbb + j;
      if (kb < nkb) {
        const uint4 cur0 = wb[j][0], cur1 = wb[j][1], cur2 = wb[j][2], cur3 = wb[j][3];
        const int kn = kb + W8_PD;
        if (kn < nkb) {
          wb[j][0] = ldg_stream(wp0 + (size_t)kn * 1024);
          wb[j][1] = ldg_stream(wp0 + (size_t)kn * 1024 + 512);
          wb[j][2] = ldg_stream(wp1 + (size_t)kn * 1024);
          wb[j][3] = ldg_stream(wp1 + (size_t)kn * 1024 + 512);
        }
        uint4 xa[MT], xb[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const uint32_t a = xs_base + (uint32_t)((t * 8 * xstride + kb * 64) * 2);
          xa[t] = lds128(a);
          xb[t] = lds128(a + 16);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
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
            const uint4& xv = (i < 2) ? xa[t] : xb[t];
            const uint32_t b0 = (i & 1) ? xv.z : xv.x;
            const uint32_t b1 = (i & 1) ? xv.w : xv.y;
            mma_f16_16816(acc[0][t], r0a0, r0a1, r0a2, r0a3, b0, b1);
            mma_f16_16816(acc[1][t], r1a0, r1a1, r1a2, r1a3, b0, b1);
          }
        }
      }
    }
  }

  // 4) partial tile -> shared (aliases the activation tile)
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

  // 5) epilogue: items are (row, 128-channel group); a warp owns an item,
  //    a lane owns 4 consecutive channels.  Rank r of the cluster takes items
  //    r, r+S, ... and sums the S partials in rank order.
  const int groups = (MODE == kSiluMul) ? 1 : 2;
  const int items = p.M * groups;
  for (int it = split + S * warp; it < items; it += S * W8_WARPS) {
    const int m = it / groups;
    const int grp = it - m * groups;
    float v[4], u[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) { v[e] = 0.f; u[e] = 0.f; }
    const int ch0 = grp * 128 + lane * 4;
    for (int s = 0; s < S; ++s) {
      const float* rr = (S > 1) ? cluster.map_shared_rank(red, s) : red;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[e] += rr[(ch0 + e) * RS + m];
        if (MODE == kSiluMul) u[e] += rr[(ch0 + 128 + e) * RS + m];
      }
    }
    const int gch = tile * W8_NT + ch0;  // global output channel of v[0]
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] *= __ldg(p.scale + gch + e);

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
      if (lane == 0) p.hstat_out[(size_t)(gch / 128) * p.M + m] = ss;
    } else if (MODE == kSiluMul) {
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float gv = v[e];
        const float uv = u[e] * __ldg(p.scale + gch + 128 + e);
        o[e] = (gv / (1.0f + expf(-gv))) * uv;
      }
      uint2 pk;
      pk.x = pack_f16x2(o[0], o[1]);
      pk.y = pack_f16x2(o[2], o[3]);
      *reinterpret_cast<uint2*>(p.act + (size_t)m * (p.N / 2) + tile * 128 + lane * 4) = pk;
    } else {  // kQKV
      const int head = gch / 128;
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

// ------------------------------------------------------------------ repack
// dst row-block = (src_rb / grp) * gstride + src_rb % grp + base
__global__ void w8_repack_kernel(const int8_t* __restrict__ src, int n_src, int K,
                                 uint8_t* __restrict__ dst, int grp, int gstride, int base) {
  const size_t nchunks = (size_t)(n_src / 16) * (K / 64) * 64;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < nchunks;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int lane = idx & 31;
    const int half = (idx >> 5) & 1;
    const size_t rest = idx >> 6;
    const int kb = rest % (K / 64);
    const int rb = rest / (K / 64);
    const int row = rb * 16 + (lane >> 2) + half * 8;
    const int col = kb * 64 + 16 * (lane & 3);
    uint4 v = *reinterpret_cast<const uint4*>(src + (size_t)row * K + col);
    v.x ^= 0x80808080u; v.y ^= 0x80808080u; v.z ^= 0x80808080u; v.w ^= 0x80808080u;
    const int drb = (rb / grp) * gstride + rb % grp + base;
    *reinterpret_cast<uint4*>(dst + w8_packed_offset(drb, kb, half, lane, K)) = v;
  }
}

__global__ void w8_scale_kernel(const __half* __restrict__ s, int n_src, float* __restrict__ dst,
                                int grp, int gstride, int base) {
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= n_src) return;
  const int rb = ch >> 4;
  const int drb = (rb / grp) * gstride + rb % grp + base;
  dst[drb * 16 + (ch & 15)] = __half2float(s[ch]);
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
template <int MT, int MODE, int XSRC>
static cudaError_t launch_mt(const W8Params& p, size_t smem, cudaStream_t st) {
  auto kern = w8_gemm_kernel<MT, MODE, XSRC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if (p.splits > 8) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
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

template <int MODE, int XSRC>
static cudaError_t launch_mode(const W8Params& p, size_t smem, cudaStream_t st) {
  if (p.M <= 8) return launch_mt<1, MODE, XSRC>(p, smem, st);
  if (p.M <= 16) return launch_mt<2, MODE, XSRC>(p, smem, st);
  if (p.M <= 32) return launch_mt<4, MODE, XSRC>(p, smem, st);
  return launch_mt<8, MODE, XSRC>(p, smem, st);
}

int w8_pick_splits(int N, int K, int M, int num_sms, int max_splits) {
  const int tiles = N / W8_NT;
  const int nkb = K / 64;
  const int mp = M <= 8 ? 8 : (M <= 16 ? 16 : (M <= 32 ? 32 : 64));
  int s = 1;
  // grow the cluster until the grid covers two CTAs per SM and the activation
  // slice stays small enough for two CTAs per SM
  while (s < max_splits && nkb / (s * 2) >= 2 &&
         (tiles * s < 2 * num_sms || (size_t)mp * (nkb / s * 64 + 8) * 2 > 96 * 1024))
    s *= 2;
  return s;
}

size_t w8_smem_bytes(const W8Params& p) {
  const int mp = p.M <= 8 ? 8 : (p.M <= 16 ? 16 : (p.M <= 32 ? 32 : 64));
  const int nkb_all = p.K / 64;
  int max_nkb = 0;
  for (int s = 0; s < p.splits; ++s) {
    const int n = (s + 1) * nkb_all / p.splits - s * nkb_all / p.splits;
    if (n > max_nkb) max_nkb = n;
  }
  const size_t xs = (size_t)mp * (max_nkb * 64 + 8) * 2 + mp * 4;
  const size_t red = (size_t)W8_NT * (mp + 1) * 4;
  return xs > red ? xs : red;
}

static cudaError_t w8_gemm_launch_once(const W8Params& p, int mode, int xsrc, cudaStream_t st) {
  const size_t smem = w8_smem_bytes(p);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (mode == kQKV && xsrc == kXHNorm) return launch_mode<kQKV, kXHNorm>(p, smem, st);
  if (mode == kResid && xsrc == kXF16) return launch_mode<kResid, kXF16>(p, smem, st);
  if (mode == kSiluMul && xsrc == kXHNorm) return launch_mode<kSiluMul, kXHNorm>(p, smem, st);
  if (mode == kStore && xsrc == kXF16) return launch_mode<kStore, kXF16>(p, smem, st);
  if (mode == kStore && xsrc == kXHNorm) return launch_mode<kStore, kXHNorm>(p, smem, st);
  return cudaErrorInvalidValue;
}

cudaError_t w8_gemm_launch(const W8Params& p, int mode, int xsrc, cudaStream_t st) {
  if (p.M < 1 || p.M > 64 || p.N % W8_NT || p.K % 64 || p.splits < 1 || p.splits > 16 ||
      p.K / 64 < p.splits)
    return cudaErrorInvalidValue;
  // a cluster that cannot be scheduled (too large for a GPC at this
  // footprint) is retried with half the split
  W8Params q = p;
  for (;;) {
    cudaError_t e = w8_gemm_launch_once(q, mode, xsrc, st);
    if (e == cudaSuccess || q.splits == 1 ||
        (e != cudaErrorInvalidClusterSize && e != cudaErrorLaunchOutOfResources))
      return e;
    (void)cudaGetLastError();
    q.splits /= 2;
  }
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
