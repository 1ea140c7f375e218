// Tied lm_head + greedy argmax + longest-prefix acceptance.
//
// logits[m, v] = hn[m, :] . E[v, :]  for the block rows, never materialised:
// each CTA streams a contiguous slice of the bf16 vocabulary matrix E [V, H]
// (1.56 GB at the 27B dims) straight from HBM into registers and keeps only a
// running (max, index) per block row (generate.py:604-605, dflash.py:133-136).
//
// MMA: mma.sync m16n8k16 bf16 with swap-AB (16 vocab rows x 8 block rows per
// op).  K is consumed in a lane-permuted order so every operand load is one
// 16-byte vector load of 8 consecutive bf16: lane c of a quad holds
// k = 8c..8c+7 of a 32-wide block, which the two MMAs of that block treat as
// logical k {2c, 2c+1, 2c+8, 2c+9}.  The same permutation applied to E and to
// hn leaves every dot product unchanged.
//
// Ties: the smallest vocabulary index among equal maxima wins, like the
// strict '>' scan of the reference's CPU argmax (ane/src/wrapper.rs:108-140)
// and numpy/MLX argmax.  NaN logits never win.
#include "kernels.cuh"

namespace dfl {

constexpr int LM_WARPS = 8;


__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return (v > bv) || (v == bv && i < bi);
}

constexpr int LM_PD = 3;          // k32 blocks of E in flight per warp
constexpr int LM_CHK = 256;       // hn k per ring stage
constexpr int LM_NST = 3;
constexpr int LM_LD = LM_CHK + 32;  // bf16 per staged row (+64 B: conflict-free 16-byte reads)

template <int MT>
__global__ void __launch_bounds__(LM_WARPS * 32, 2) lm_argmax_kernel(const LmParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int MP = MT * 8;
  __nv_bfloat16* ring = reinterpret_cast<__nv_bfloat16*>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int units = (p.V + 31) / 32;  // 32 vocab rows per warp-unit
  const int u0 = (int)((long long)blockIdx.x * units / gridDim.x);
  const int u1 = (int)((long long)(blockIdx.x + 1) * units / gridDim.x);
  const int rounds = (u1 - u0 + LM_WARPS - 1) / LM_WARPS;
  const int nk32 = p.H / 32;
  const int nchunks = (p.H + LM_CHK - 1) / LM_CHK;
  const int total_chunks = rounds * nchunks;

  // hn ring: global chunk gq = round * nchunks + q holds hn[0..MP)[q*CHK, +CHK)
  auto load_chunk = [&](int gq) {
    if (gq < total_chunks) {
      __nv_bfloat16* st = ring + (size_t)(gq % LM_NST) * MP * LM_LD;
      const int k0 = (gq % nchunks) * LM_CHK;
      const int cpr = min(LM_CHK, p.H - k0) / 8;
      for (int idx = threadIdx.x; idx < MP * cpr; idx += LM_WARPS * 32) {
        const int m = idx / cpr, kk = (idx - m * cpr) * 8;
        const bool ok = m < p.M;
        cp_async16_zfill(smem_u32(st + m * LM_LD + kk), p.hn + (size_t)(ok ? m : 0) * p.H + k0 + kk, ok);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int q = 0; q < LM_NST - 1; ++q) load_chunk(q);

  // running best for columns (t*8 + 2c + e), identical in the 8 lanes of a column quad
  float bv[MT][2];
  int bi[MT][2];
#pragma unroll
  for (int t = 0; t < MT; ++t)
#pragma unroll
    for (int e = 0; e < 2; ++e) { bv[t][e] = -INFINITY; bi[t][e] = 0x7fffffff; }

  const uint32_t ring_lane = smem_u32(ring) + (uint32_t)((g * LM_LD + 8 * c) * 2);
  constexpr int K32_PER_CHUNK = LM_CHK / 32;
  for (int rd = 0; rd < rounds; ++rd) {
    const int u = u0 + rd * LM_WARPS + warp;
    const bool active = u < u1;
    const int vbase = u * 32;
    // rows vbase + {g, g+8, 16+g, 24+g}; rows >= V clamp to V-1 (masked below)
    const __nv_bfloat16* er[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      int v = vbase + (r >> 1) * 16 + (r & 1) * 8 + g;
      v = v < p.V ? v : p.V - 1;
      er[r] = p.E + (size_t)v * p.H + 8 * c;
    }
    float acc[2][MT][4];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[r][t][e] = 0.f;
    uint4 wb[LM_PD][4];
    if (active) {
#pragma unroll
      for (int j = 0; j < LM_PD; ++j)
        if (j < nk32)
#pragma unroll
          for (int r = 0; r < 4; ++r) wb[j][r] = ldg_stream(er[r] + j * 32);
    }
    for (int kb = 0; kb < nk32; kb += LM_PD) {
#pragma unroll
      for (int j = 0; j < LM_PD; ++j) {
        const int k = kb + j;
        if (k < nk32) {
          if (k % K32_PER_CHUNK == 0) {  // uniform across the CTA
            cp_async_wait<LM_NST - 2>();
            __syncthreads();
            load_chunk(rd * nchunks + k / K32_PER_CHUNK + LM_NST - 1);
          }
          if (active) {
            uint4 cur[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) cur[r] = wb[j][r];
            if (k + LM_PD < nk32)
#pragma unroll
              for (int r = 0; r < 4; ++r) wb[j][r] = ldg_stream(er[r] + (k + LM_PD) * 32);
            const int gq = rd * nchunks + k / K32_PER_CHUNK;
            const uint32_t kaddr = ring_lane +
                (uint32_t)(((gq % LM_NST) * MP * LM_LD + (k % K32_PER_CHUNK) * 32) * 2);
#pragma unroll
            for (int t = 0; t < MT; ++t) {
              uint4 hv;
              asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                           : "=r"(hv.x), "=r"(hv.y), "=r"(hv.z), "=r"(hv.w)
                           : "r"(kaddr + (uint32_t)(t * 8 * LM_LD * 2)));
              // MMA 0: phys k 8c..8c+3 ; MMA 1: 8c+4..8c+7
#pragma unroll
              for (int r = 0; r < 2; ++r) {
                mma_bf16_16816(acc[r][t], cur[2 * r].x, cur[2 * r + 1].x, cur[2 * r].y,
                               cur[2 * r + 1].y, hv.x, hv.y);
                mma_bf16_16816(acc[r][t], cur[2 * r].z, cur[2 * r + 1].z, cur[2 * r].w,
                               cur[2 * r + 1].w, hv.z, hv.w);
              }
            }
          }
        }
      }
    }
    if (active) {
      // candidates of this unit -> running best
#pragma unroll
      for (int t = 0; t < MT; ++t) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float v = -INFINITY;
          int idx = 0x7fffffff;
#pragma unroll
          for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int hgh = 0; hgh < 2; ++hgh) {
              const int vi = vbase + r * 16 + hgh * 8 + g;
              float x = acc[r][t][hgh * 2 + e];
              if (x != x) x = -INFINITY;
              if (vi < p.V && better(x, vi, v, idx)) { v = x; idx = vi; }
            }
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
            if (better(ov, oi, v, idx)) { v = ov; idx = oi; }
          }
          if (better(v, idx, bv[t][e], bi[t][e])) { bv[t][e] = v; bi[t][e] = idx; }
        }
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // CTA reduction across warps (reuses the ring)
  float* sv = reinterpret_cast<float*>(smem);
  int* si = reinterpret_cast<int*>(sv + LM_WARPS * MP);
  if (g == 0) {
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sv[warp * MP + t * 8 + 2 * c + e] = bv[t][e];
        si[warp * MP + t * 8 + 2 * c + e] = bi[t][e];
      }
  }
  __syncthreads();
  for (int m = threadIdx.x; m < p.M; m += blockDim.x) {
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int w = 0; w < LM_WARPS; ++w)
      if (better(sv[w * MP + m], si[w * MP + m], v, idx)) { v = sv[w * MP + m]; idx = si[w * MP + m]; }
    p.best_val[(size_t)blockIdx.x * p.M + m] = v;
    p.best_idx[(size_t)blockIdx.x * p.M + m] = idx;
  }
}

// One CTA per sequence, one warp per block row: combine the per-CTA partials
// of rows 1..B-1 into the draft tokens, then (if target tokens are given) the
// longest matching prefix and the correction token (generate.py:722-728).
__global__ void argmax_accept_kernel(const float* __restrict__ best_val,
                                     const int* __restrict__ best_idx, int nparts, int M, int block,
                                     int32_t* __restrict__ out_tokens,
                                     const int32_t* __restrict__ target, int32_t* __restrict__ acc_len,
                                     int32_t* __restrict__ correction) {
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int toks[1024];
  for (int j = 1 + warp; j < block; j += blockDim.x >> 5) {
    const int m = b * block + j;
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int q = lane; q < nparts; q += 32) {
      const float x = best_val[(size_t)q * M + m];
      const int i = best_idx[(size_t)q * M + m];
      if (better(x, i, v, idx)) { v = x; idx = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (better(ov, oi, v, idx)) { v = ov; idx = oi; }
    }
    if (lane == 0) {
      if (idx == 0x7fffffff) idx = 0;  // every logit NaN: id 0, like a strict '>' scan
      toks[j - 1] = idx;
      if (out_tokens) out_tokens[(size_t)b * (block - 1) + j - 1] = idx;
    }
  }
  __syncthreads();
  if (target && threadIdx.x == 0) {
    const int32_t* t = target + (size_t)b * block;
    int a = 0;
    while (a < block - 1 && toks[a] == t[a]) ++a;
    acc_len[b] = a;
    correction[b] = t[a];
  }
}

// Standalone acceptance for caller-supplied draft tokens.
__global__ void accept_kernel(const int32_t* __restrict__ draft, const int32_t* __restrict__ target,
                              int batch, int block, int32_t* __restrict__ acc_len,
                              int32_t* __restrict__ correction) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const int32_t* d = draft + (size_t)b * (block - 1);
  const int32_t* t = target + (size_t)b * block;
  int a = 0;
  while (a < block - 1 && d[a] == t[a]) ++a;
  acc_len[b] = a;
  correction[b] = t[a];
}

template <int MT>
static cudaError_t lm_launch_t(const LmParams& p, int grid, cudaStream_t st) {
  const size_t ring = (size_t)LM_NST * MT * 8 * LM_LD * 2;
  const size_t red = (size_t)LM_WARPS * MT * 8 * 8;
  const size_t smem = ring > red ? ring : red;
  cudaError_t e = cudaFuncSetAttribute(lm_argmax_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  lm_argmax_kernel<MT><<<grid, LM_WARPS * 32, smem, st>>>(p);
  return cudaGetLastError();
}

cudaError_t lm_argmax_launch(const LmParams& p, int grid, cudaStream_t st) {
  if (p.H % 32 || p.M < 1 || p.M > 64 || p.V < 1) return cudaErrorInvalidValue;
  const int mt = (p.M + 7) / 8;
  if (mt == 1) return lm_launch_t<1>(p, grid, st);
  if (mt == 2) return lm_launch_t<2>(p, grid, st);
  if (mt <= 4) return lm_launch_t<4>(p, grid, st);
  return lm_launch_t<8>(p, grid, st);
}

cudaError_t argmax_accept_launch(const float* bv, const int* bi, int nparts, int M, int block,
                                 int batch, int32_t* out_tokens, const int32_t* target,
                                 int32_t* acc_len, int32_t* correction, cudaStream_t st) {
  if (block < 2 || block > 1024) return cudaErrorInvalidValue;
  argmax_accept_kernel<<<batch, 32 * (block - 1 < 32 ? block - 1 : 32), 0, st>>>(
      bv, bi, nparts, M, block, out_tokens, target, acc_len, correction);
  return cudaGetLastError();
}

cudaError_t accept_launch(const int32_t* draft, const int32_t* target, int batch, int block,
                          int32_t* acc_len, int32_t* correction, cudaStream_t st) {
  if (block < 2 || batch < 1) return cudaErrorInvalidValue;
  accept_kernel<<<(batch + 127) / 128, 128, 0, st>>>(draft, target, batch, block, acc_len, correction);
  return cudaGetLastError();
}

}  // namespace dfl
