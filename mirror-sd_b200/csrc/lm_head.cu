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

template <int MT>
__global__ void __launch_bounds__(LM_WARPS * 32) lm_argmax_kernel(const LmParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int units = (p.V + 31) / 32;  // 32 vocab rows per warp-unit
  const int u0 = (int)((long long)blockIdx.x * units / gridDim.x);
  const int u1 = (int)((long long)(blockIdx.x + 1) * units / gridDim.x);
  const int nk32 = p.H / 32;

  // running best for columns (t*8 + 2c + e), identical in the 8 lanes of a column quad
  float bv[MT][2];
  int bi[MT][2];
#pragma unroll
  for (int t = 0; t < MT; ++t)
#pragma unroll
    for (int e = 0; e < 2; ++e) { bv[t][e] = -INFINITY; bi[t][e] = 0x7fffffff; }

  // activation row pointers (rows >= M read row 0; their results are dropped)
  const __nv_bfloat16* hrow[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const int m = t * 8 + g;
    hrow[t] = p.hn + (size_t)(m < p.M ? m : 0) * p.H + 8 * c;
  }

  for (int u = u0 + warp; u < u1; u += LM_WARPS) {
    const int vbase = u * 32;
    // rows vbase + {g, g+8, 16+g, 24+g}; rows >= V clamp to V-1 (masked below)
    const __nv_bfloat16* er[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int v = vbase + (r >> 1) * 16 + (r & 1) * 8 + g;
      er[r] = p.E + (size_t)(v < p.V ? v : p.V - 1) * p.H + 8 * c;
    }
    float acc[2][MT][4];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[r][t][e] = 0.f;

    constexpr int U = 4;  // k32 blocks in flight
    uint4 wb[U][4];
#pragma unroll
    for (int j = 0; j < U; ++j)
      if (j < nk32)
#pragma unroll
        for (int r = 0; r < 4; ++r) wb[j][r] = ldg_stream(er[r] + j * 32);
    for (int kb = 0; kb < nk32; kb += U) {
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const int k = kb + j;
        if (k < nk32) {
          uint4 cur[4];
#pragma unroll
          for (int r = 0; r < 4; ++r) cur[r] = wb[j][r];
          if (k + U < nk32)
#pragma unroll
            for (int r = 0; r < 4; ++r) wb[j][r] = ldg_stream(er[r] + (k + U) * 32);
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            const uint4 hv = __ldg(reinterpret_cast<const uint4*>(hrow[t] + k * 32));
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
            if (vi >= p.V || x != x) x = -INFINITY;
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

  // CTA reduction across warps
  __shared__ float sv[LM_WARPS][MT * 8];
  __shared__ int si[LM_WARPS][MT * 8];
  if (g == 0) {
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sv[warp][t * 8 + 2 * c + e] = bv[t][e];
        si[warp][t * 8 + 2 * c + e] = bi[t][e];
      }
  }
  __syncthreads();
  for (int m = threadIdx.x; m < p.M; m += blockDim.x) {
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int w = 0; w < LM_WARPS; ++w)
      if (better(sv[w][m], si[w][m], v, idx)) { v = sv[w][m]; idx = si[w][m]; }
    p.best_val[(size_t)blockIdx.x * p.M + m] = v;
    p.best_idx[(size_t)blockIdx.x * p.M + m] = idx;
  }
}

// One CTA per sequence: combine the per-CTA partials of rows 1..B-1 into the
// draft tokens, then (if target tokens are given) the longest matching prefix
// and the correction token (generate.py:722-728).
__global__ void argmax_accept_kernel(const float* __restrict__ best_val,
                                     const int* __restrict__ best_idx, int nparts, int M, int block,
                                     int32_t* __restrict__ out_tokens,
                                     const int32_t* __restrict__ target, int32_t* __restrict__ acc_len,
                                     int32_t* __restrict__ correction) {
  const int b = blockIdx.x;
  __shared__ int toks[1024];
  for (int j = 1 + threadIdx.x; j < block; j += blockDim.x) {
    const int m = b * block + j;
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int q = 0; q < nparts; ++q) {
      const float x = best_val[(size_t)q * M + m];
      const int i = best_idx[(size_t)q * M + m];
      if (better(x, i, v, idx)) { v = x; idx = i; }
    }
    if (idx == 0x7fffffff) idx = 0;  // every logit NaN: fall back to id 0 like a strict '>' scan
    toks[j - 1] = idx;
    if (out_tokens) out_tokens[(size_t)b * (block - 1) + j - 1] = idx;
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

cudaError_t lm_argmax_launch(const LmParams& p, int grid, cudaStream_t st) {
  if (p.H % 32 || p.M < 1 || p.M > 64 || p.V < 1) return cudaErrorInvalidValue;
  const int mt = (p.M + 7) / 8;
  if (mt == 1) lm_argmax_kernel<1><<<grid, LM_WARPS * 32, 0, st>>>(p);
  else if (mt == 2) lm_argmax_kernel<2><<<grid, LM_WARPS * 32, 0, st>>>(p);
  else if (mt <= 4) lm_argmax_kernel<4><<<grid, LM_WARPS * 32, 0, st>>>(p);
  else lm_argmax_kernel<8><<<grid, LM_WARPS * 32, 0, st>>>(p);
  return cudaGetLastError();
}

cudaError_t argmax_accept_launch(const float* bv, const int* bi, int nparts, int M, int block,
                                 int batch, int32_t* out_tokens, const int32_t* target,
                                 int32_t* acc_len, int32_t* correction, cudaStream_t st) {
  if (block < 2 || block > 1024) return cudaErrorInvalidValue;
  argmax_accept_kernel<<<batch, 128, 0, st>>>(bv, bi, nparts, M, block, out_tokens, target, acc_len,
                                              correction);
  return cudaGetLastError();
}

cudaError_t accept_launch(const int32_t* draft, const int32_t* target, int batch, int block,
                          int32_t* acc_len, int32_t* correction, cudaStream_t st) {
  if (block < 2 || batch < 1) return cudaErrorInvalidValue;
  accept_kernel<<<(batch + 127) / 128, 128, 0, st>>>(draft, target, batch, block, acc_len, correction);
  return cudaGetLastError();
}

}  // namespace dfl
