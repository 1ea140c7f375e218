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

// ---------------------------------------------------------------- tcgen05 path
// E is repacked once (lm_pack) into 128-row vocabulary tiles whose k64 blocks
// are contiguous 16 KB runs already laid out in the UMMA's 128-byte swizzle:
// [V/128][H/64][128 rows][128 B], rows >= V zero.  A CTA owns a contiguous
// range of vocabulary tiles.  warp 0 streams E blocks (cp.async.bulk) and the
// matching hn tile (TMA, 128-byte swizzle); warp 1 issues
// tcgen05.mma M=128 (vocab) x N=MP (block rows) x K=16 into one of two TMEM
// accumulators; warps 2..5 take the argmax of the other accumulator while
// the next tile streams in.
constexpr int LT_THREADS = 192;
constexpr int LT_E_BYTES = 128 * 128;
// ring depth: as many stages as about 210 KB of shared memory holds, so one
// CTA keeps enough bytes in flight to draw its share of HBM bandwidth
template <int MP>
struct LtCfg {
  static constexpr int STAGE = LT_E_BYTES + MP * 128;
  static constexpr int NS = (210 * 1024) / STAGE < 12 ? (210 * 1024) / STAGE : 12;
};

template <int MP>
__global__ void __launch_bounds__(LT_THREADS, 1)
    lm_tc_kernel(const __grid_constant__ CUtensorMap map_h, const LmParams p, const uint8_t* e_tiles,
                 int vt_total, int* err) {
  griddep_wait();
  griddep_launch_dependents();
  constexpr int H_BYTES = MP * 128;
  constexpr int STAGE = LT_E_BYTES + H_BYTES;
  static_assert(STAGE % 1024 == 0, "stage alignment");
  constexpr uint32_t ACC_COLS = MP <= 32 ? 32 : 64;
  constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int LT_NS = LtCfg<MP>::NS;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + LT_NS * STAGE);
  uint64_t* empty = full + LT_NS;
  uint64_t* acc_full = empty + LT_NS;   // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red_v = reinterpret_cast<float*>(tmem_slot + 4);   // [4][64]
  int* red_i = reinterpret_cast<int*>(red_v + 4 * 64);       // [4][64]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int VT = (p.V + 127) / 128;
  const int nkb = p.H / 64;
  // balanced contiguous ranges: every CTA owns floor or ceil(VT / grid) tiles
  const int t0 = (int)(((long long)blockIdx.x * vt_total) / gridDim.x);
  const int t1 = min(VT, (int)(((long long)(blockIdx.x + 1) * vt_total) / gridDim.x));
  const int ntile = max(0, t1 - t0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < LT_NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&map_h);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int ti = 0; ti < ntile; ++ti) {
        const uint8_t* eb = e_tiles + (size_t)(t0 + ti) * nkb * LT_E_BYTES;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % LT_NS;
          const uint32_t ph = (it / LT_NS) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, err, abort_flag)) { ti = ntile; break; }
          uint8_t* st = smem + s * STAGE;
          mbar_arrive_expect_tx(&full[s], STAGE);
          bulk_load(st, eb + (size_t)kb * LT_E_BYTES, LT_E_BYTES, &full[s]);
          tma_load_2d(st + LT_E_BYTES, &map_h, &full[s], kb * 64, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(128, MP, 1);
      int it = 0;
      bool ok = true;
      for (int ti = 0; ti < ntile && ok; ++ti) {
        const int b = ti & 1;
        if (!mbar_wait(&acc_empty[b], ((ti >> 1) & 1) ^ 1, err, abort_flag)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * ACC_COLS;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % LT_NS;
          const uint32_t ph = (it / LT_NS) & 1;
          if (!mbar_wait(&full[s], ph, err, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * STAGE);
          const uint64_t adesc = umma_desc_sw128(sa);
          const uint64_t bdesc = umma_desc_sw128(sa + LT_E_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k) umma_f16(acc, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0);
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[b]);
      }
    }
  } else {
    const int q = warp & 3;
    // running best: lane c owns columns c and c + 32
    float bv[2] = {-INFINITY, -INFINITY};
    int bi[2] = {0x7fffffff, 0x7fffffff};
    for (int ti = 0; ti < ntile; ++ti) {
      const int b = ti & 1;
      if (!mbar_wait(&acc_full[b], (ti >> 1) & 1, err, abort_flag)) break;
      tc_fence_after();
      const int vrow = (t0 + ti) * 128 + q * 32 + lane;
      const bool vok = vrow < p.V;
#pragma unroll
      for (int c0 = 0; c0 < MP; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + b * ACC_COLS + ((uint32_t)(q * 32) << 16) + c0, r);
        tmem_ld_wait();
        if (c0 + 32 >= MP) {  // last chunk: hand the accumulator back before the shuffles
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          if (c0 + c < MP) {
            float v = __uint_as_float(r[c]);
            int idx = vrow;
            if (!vok || v != v) { v = -INFINITY; idx = 0x7fffffff; }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
              const float ov = __shfl_xor_sync(0xffffffffu, v, o);
              const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
              if (better(ov, oi, v, idx)) { v = ov; idx = oi; }
            }
            if (lane == c && better(v, idx, bv[c0 / 32], bi[c0 / 32])) {
              bv[c0 / 32] = v;
              bi[c0 / 32] = idx;
            }
          }
        }
      }
    }
    red_v[q * 64 + lane] = bv[0];
    red_i[q * 64 + lane] = bi[0];
    red_v[q * 64 + 32 + lane] = bv[1];
    red_i[q * 64 + 32 + lane] = bi[1];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  for (int m = threadIdx.x; m < p.M; m += LT_THREADS) {
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int w = 0; w < 4; ++w)
      if (better(red_v[w * 64 + m], red_i[w * 64 + m], v, idx)) { v = red_v[w * 64 + m]; idx = red_i[w * 64 + m]; }
    p.best_val[(size_t)blockIdx.x * p.M + m] = v;
    p.best_idx[(size_t)blockIdx.x * p.M + m] = idx;
  }
}

// E [V, H] bf16 row-major -> [ceil(V/128)][H/64][128 rows][128 B] in the
// 128-byte swizzle (16-byte chunk j of row r stored at chunk j ^ (r % 8)).
__global__ void lm_pack_kernel(const __nv_bfloat16* __restrict__ E, int V, int H, uint8_t* __restrict__ out) {
  const int nkb = H / 64;
  const int VT = (V + 127) / 128;
  const size_t total = (size_t)VT * nkb * 128 * 8;  // 16-byte chunks
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int j = idx & 7;
    const int r = (idx >> 3) & 127;
    const size_t rest = idx >> 10;
    const int kb = rest % nkb;
    const int vt = rest / nkb;
    const int v = vt * 128 + r;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (v < V) val = *reinterpret_cast<const uint4*>(E + (size_t)v * H + kb * 64 + j * 8);
    *reinterpret_cast<uint4*>(out + (((size_t)vt * nkb + kb) * 128 + r) * 128 + ((j ^ (r & 7)) << 4)) = val;
  }
}

// One CTA per sequence, one warp per block row: combine the per-CTA partials
// of rows 1..B-1 into the draft tokens, then (if target tokens are given) the
// longest matching prefix and the correction token (generate.py:722-728).
__global__ void argmax_accept_kernel(const float* __restrict__ best_val,
                                     const int* __restrict__ best_idx, int nparts, int M, int block,
                                     int first, int32_t* __restrict__ out_tokens,
                                     const int32_t* __restrict__ target, int32_t* __restrict__ acc_len,
                                     int32_t* __restrict__ correction) {
  griddep_wait();
  griddep_launch_dependents();
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int toks[1024];
  for (int j = 1 + warp; j < block; j += blockDim.x >> 5) {
    const int m = b * (block - first) + j - first;   // partial row (rows j < first are absent)
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

typedef CUresult (*EncodeTiledFn3)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static bool map_rows_sw128(CUtensorMap* m, const void* base, uint64_t K, uint64_t rows, uint32_t box_rows) {
  static EncodeTiledFn3 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return false;
    fn = reinterpret_cast<EncodeTiledFn3>(ptr);
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (K * 2) % 16) return false;
  cuuint64_t dims[2] = {K, rows};
  cuuint64_t strides[1] = {K * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// CTAs: as few as keep the per-CTA tile count at ceil(VT / SMs) (132 of 148
// SMs for the 1187 tiles of a 151936 vocabulary; measured faster than
// spreading 8-9 tiles over all 148 SMs at both 4096 and 5120 hidden)
int lm_grid(int V, int num_sms) {
  const int VT = (V + 127) / 128;
  const int per = (VT + num_sms - 1) / num_sms;
  return (VT + per - 1) / per;
}

template <int MP>
static cudaError_t lm_tc_t(const CUtensorMap& mh, const LmParams& p, const uint8_t* et, int grid,
                           int vt_total, int* err, cudaStream_t st) {
  const size_t smem = (size_t)LtCfg<MP>::NS * LtCfg<MP>::STAGE + 1024 + 256 + 8 * 64 * 4;
  cudaError_t e = cudaFuncSetAttribute(lm_tc_kernel<MP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  DFL_TRY(max_smem_carveout(lm_tc_kernel<MP>));
  return launch_pdl(lm_tc_kernel<MP>, dim3(grid), dim3(LT_THREADS), smem, st, mh, p, et, vt_total, err);
}

// returns the grid used (partials written for that many CTAs) via *grid_out
cudaError_t lm_argmax_launch(const LmParams& p, const uint8_t* e_tiles, int num_sms, int* err,
                             int* grid_out, cudaStream_t st) {
  if (p.H % 64 || p.M < 1 || p.M > 64 || p.V < 1) return cudaErrorInvalidValue;
  const int VT = (p.V + 127) / 128;
  const int grid = lm_grid(p.V, num_sms);
  *grid_out = grid;
  const int mp = (p.M + 15) / 16 * 16;
  CUtensorMap mh;
  if (!map_rows_sw128(&mh, p.hn, p.H, p.M, mp)) return cudaErrorInvalidValue;
  if (mp == 16) return lm_tc_t<16>(mh, p, e_tiles, grid, VT, err, st);
  if (mp == 32) return lm_tc_t<32>(mh, p, e_tiles, grid, VT, err, st);
  if (mp == 48) return lm_tc_t<48>(mh, p, e_tiles, grid, VT, err, st);
  return lm_tc_t<64>(mh, p, e_tiles, grid, VT, err, st);
}

size_t lm_pack_bytes(int V, int H) { return (size_t)((V + 127) / 128) * 128 * H * 2; }

cudaError_t lm_pack_launch(const __nv_bfloat16* E, int V, int H, uint8_t* out, cudaStream_t st) {
  if (H % 64 || V < 1) return cudaErrorInvalidValue;
  lm_pack_kernel<<<2048, 256, 0, st>>>(E, V, H, out);
  return cudaGetLastError();
}

cudaError_t argmax_accept_launch(const float* bv, const int* bi, int nparts, int M, int block,
                                 int batch, int32_t* out_tokens, const int32_t* target,
                                 int32_t* acc_len, int32_t* correction, cudaStream_t st, int first) {
  if (block < 2 || block > 1024 || first < 0 || first > 1) return cudaErrorInvalidValue;
  DFL_TRY(max_smem_carveout(argmax_accept_kernel));
  return launch_pdl(argmax_accept_kernel, dim3(batch), dim3(32 * (block - 1 < 32 ? block - 1 : 32)), 0,
                    st, bv, bi, nparts, M, block, first, out_tokens, target, acc_len, correction);
}

cudaError_t accept_launch(const int32_t* draft, const int32_t* target, int batch, int block,
                          int32_t* acc_len, int32_t* correction, cudaStream_t st) {
  if (block < 2 || batch < 1) return cudaErrorInvalidValue;
  DFL_TRY(max_smem_carveout(accept_kernel));
  accept_kernel<<<(batch + 127) / 128, 128, 0, st>>>(draft, target, batch, block, acc_len, correction);
  return cudaGetLastError();
}

}  // namespace dfl
