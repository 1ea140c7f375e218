// W8A16 skinny GEMM on the 5th-gen tensor cores (tcgen05 + TMA), for the
// block rows of the draft forward (q|k|v, o, gate|up, down projections).
//
//   Y[m, n] = scale[n] * sum_k X[m, k] * Wq[n, k]      m < M <= 64, Wq int8
//
// Swap-AB: the 128 output channels of a tile are the UMMA M dimension and the
// (padded) activation rows are N (16..64), so one tcgen05.mma.kind::f16
// M=128 N=MP K=16 covers a whole tile.  Per k64 step:
//   warp 0      TMA: int8 weight tile [128 x 64 B] (row-major, no swizzle) and
//               the f16 activation tile [MP x 64] (128-byte swizzle)
//   warps 2..5  dequantise the int8 tile into a 128-byte-swizzled f16 tile
//               (one channel row per thread: PRMT with 0x6464 builds 1024+u,
//               one f16x2 subtract recovers q exactly), fence.proxy.async,
//               then arrive on the stage's "converted" barrier
//   warp 1      single-thread UMMA issue into a 128 x MP fp32 TMEM accumulator,
//               tcgen05.commit frees the stage
// The fp16 per-channel scale is applied in the epilogue (int8 values are exact
// in f16, so the product is the reference's q * s up to fp32 rounding).
// K is split over a thread-block cluster (<= 8 CTAs); partial tiles are
// reduced through distributed shared memory in rank order and the fused
// epilogues of w8_gemm.cuh run (kStore / kQKV / kResid / kSiluMul).
// Every mbarrier wait is bounded; a timeout raises the device error word and
// the CTA unwinds (TMEM released on every path).
#include <cooperative_groups.h>

#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace dfl {

constexpr int WT_NS = 3;          // pipeline stages
constexpr int WT_THREADS = 192;   // 6 warps
constexpr int WT_W8_BYTES = 128 * 64;
constexpr int WT_WF_BYTES = 128 * 128;

__device__ __forceinline__ uint4 lds128_u(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts128_u(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// 16 int8 -> 16 f16 (exact); x ^ 0x80 biases to u = q + 128
__device__ __forceinline__ void i8x16_to_f16x16(uint4 v, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u, v.w ^ 0x80808080u};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = u8x2_to_f16x2(w[i], 0x5140);
    o[2 * i + 1] = u8x2_to_f16x2(w[i], 0x5342);
  }
  lo = make_uint4(o[0], o[1], o[2], o[3]);
  hi = make_uint4(o[4], o[5], o[6], o[7]);
}

__device__ __forceinline__ void rope_lane_t(float (&y)[4], int lane, const float2* __restrict__ cs_row) {
  float z[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) z[e] = __shfl_xor_sync(0xffffffffu, y[e], 16);
  const bool lo = lane < 16;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = __ldg(cs_row + (lane & 15) * 4 + e);
    y[e] = lo ? (y[e] * t.x - z[e] * t.y) : (z[e] * t.y + y[e] * t.x);
  }
}

struct W8TcArgs {
  W8Params p;
  const int8_t* w_tiles;  // [N/128][K/64][128 rows][64 B]
  int* err;
};

template <int MP, int MODE>
__global__ void __launch_bounds__(WT_THREADS, 1)
    w8tc_kernel(const __grid_constant__ CUtensorMap map_x, const W8TcArgs args) {
  const W8Params& p = args.p;
  constexpr int X_BYTES = MP * 128;
  constexpr int STAGE = WT_WF_BYTES + X_BYTES + WT_W8_BYTES;  // multiple of 1024
  static_assert(STAGE % 1024 == 0, "stage must keep 1024-byte alignment");
  constexpr uint32_t TMEM_COLS = MP <= 32 ? 32 : 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + WT_NS * STAGE);
  uint64_t* conv = full + WT_NS;
  uint64_t* empty = conv + WT_NS;
  uint64_t* accum = empty + WT_NS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int S = p.splits;
  const int tile = blockIdx.x / S;
  const int split = blockIdx.x % S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb_all = p.K / 64;
  const int kb0 = split * nkb_all / S;
  const int nkb = (split + 1) * nkb_all / S - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < WT_NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&map_x);
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
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % WT_NS;
        const uint32_t ph = (kb / WT_NS) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, args.err, abort_flag)) break;
        uint8_t* st = smem + s * STAGE;
        mbar_arrive_expect_tx(&full[s], WT_W8_BYTES + X_BYTES);
        // the tile's k64 block is one contiguous 8 KB run of the packed weights
        bulk_load(st + WT_WF_BYTES + X_BYTES,
                  args.w_tiles + ((size_t)tile * nkb_all + kb0 + kb) * WT_W8_BYTES, WT_W8_BYTES, &full[s]);
        tma_load_2d(st + WT_WF_BYTES, &map_x, &full[s], (kb0 + kb) * 64, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(128, MP, 0);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % WT_NS;
        const uint32_t ph = (kb / WT_NS) & 1;
        if (!mbar_wait(&conv[s], ph, args.err, abort_flag)) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * STAGE);
        const uint64_t adesc = umma_desc_sw128(sa);
        const uint64_t bdesc = umma_desc_sw128(sa + WT_WF_BYTES);
#pragma unroll
        for (int k = 0; k < 4; ++k) umma_f16(tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0);
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
    }
  } else {
    // converters: piece c = 128*i + t is 16 int8 of row c/4, k 16*(c%4) .. +15;
    // reads are consecutive 16-byte pieces and the two 16-byte f16 writes of a
    // quarter-warp land on 8 distinct swizzled slots: no bank conflicts.
    const int t = threadIdx.x - 64;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % WT_NS;
      const uint32_t ph = (kb / WT_NS) & 1;
      if (!mbar_wait(&full[s], ph, args.err, abort_flag)) break;
      const uint32_t st = smem_u32(smem + s * STAGE);
      const uint32_t src = st + WT_WF_BYTES + X_BYTES;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = i * 128 + t;
        const int r = c >> 2, ch = c & 3;
        uint4 lo, hi;
        i8x16_to_f16x16(lds128_u(src + c * 16), lo, hi);
        const uint32_t dst = st + r * 128;
        sts128_u(dst + (((2 * ch) ^ (r & 7)) << 4), lo);
        sts128_u(dst + (((2 * ch + 1) ^ (r & 7)) << 4), hi);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[s]);
    }
  }

  // ---- accumulator -> shared partial tile red[128 ch][MP + 1]
  constexpr int RS = MP + 1;
  float* red = reinterpret_cast<float*>(smem);
  bool ok = true;
  if (warp >= 2) {
    ok = mbar_wait(accum, 0, args.err, abort_flag) && !*abort_flag;
    tc_fence_after();
  }
  __syncthreads();  // every warp is past the main loop: the stage memory can be reused
  if (warp >= 2 && ok) {
    const int q = warp & 3;
    const int ch = q * 32 + lane;
    const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll
    for (int c0 = 0; c0 < MP; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + c0, r);
      tmem_ld_wait();
#pragma unroll
      for (int m = 0; m < 32; ++m)
        if (c0 + m < MP) red[ch * RS + c0 + m] = __uint_as_float(r[m]);
    }
  }
  tc_fence_before();
  cg::cluster_group cluster = cg::this_cluster();
  if (S > 1) cluster.sync(); else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }

  // ---- epilogue: one item per activation row; rank r takes rows r, r+S, ...
  constexpr int NW = WT_THREADS / 32;
  constexpr int EPC = (MODE == kSiluMul) ? 2 : 4;
  const bool all_ok = !*abort_flag;
  for (int m = split + S * warp; all_ok && m < p.M; m += S * NW) {
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
    const int gch = tile * 128 + ch0;
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
        rope_lane_t(v, lane, p.rope + (size_t)(p.kv_row0 + j) * 64);
      }
      uint2 o;
      o.x = pack_f16x2(v[0], v[1]);
      o.y = pack_f16x2(v[2], v[3]);
      __half* dstp;
      if (is_q) {
        dstp = p.q_out + (((size_t)bi * p.n_q_heads + head) * p.block + j) * 128;
      } else {
        const int kvh = is_k ? head - p.n_q_heads : head - p.n_q_heads - p.n_kv_heads;
        __half* base = is_k ? p.k_out : p.v_out;
        dstp = base + (((size_t)bi * p.n_kv_heads + kvh) * p.kv_rows + p.kv_row0 + j) * 128;
      }
      *reinterpret_cast<uint2*>(dstp + lane * 4) = o;
    }
  }
  if (S > 1) cluster.sync();
}

// ------------------------------------------------------------------ tile packing
// Source row r (int8 [n_src, K] row-major) becomes output channel
// d = (r / grp) * gstride + r % grp + base (concatenation / gate|up interleave)
// and is stored tile-major: [d / 128][kb][d % 128][64 B], so the 8 KB of
// every (128-channel tile, k64) block is contiguous.
__global__ void w8_tilepack_kernel(const int8_t* __restrict__ src, int n_src, int K,
                                   int8_t* __restrict__ dst, int grp, int gstride, int base) {
  const int cpr = K / 16;
  const int nkb = K / 64;
  const size_t total = (size_t)n_src * cpr;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int r = idx / cpr, c = idx % cpr;
    const int d = (r / grp) * gstride + r % grp + base;
    const int kb = c / 4, piece = c % 4;
    const size_t off = (((size_t)(d / 128) * nkb + kb) * 128 + d % 128) * 64 + piece * 16;
    *reinterpret_cast<uint4*>(dst + off) = reinterpret_cast<const uint4*>(src + (size_t)r * K)[c];
  }
}

// ------------------------------------------------------------------ host
typedef CUresult (*EncodeTiledFn2)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn2 encode_fn() {
  static EncodeTiledFn2 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn2>(ptr);
  }
  return fn;
}

static bool map2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize, uint64_t inner,
                  uint64_t outer, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  EncodeTiledFn2 enc = encode_fn();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15) || (inner * esize) % 16) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * esize};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MP, int MODE>
static cudaError_t w8tc_launch_t(const CUtensorMap& mx, const W8TcArgs& a, cudaStream_t st) {
  constexpr size_t STAGE = WT_WF_BYTES + MP * 128 + WT_W8_BYTES;
  const size_t smem = WT_NS * STAGE + 1024 + 256;
  auto kern = w8tc_kernel<MP, MODE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.p.N / 128) * a.p.splits);
  cfg.blockDim = dim3(WT_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.p.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, mx, a);
}

template <int MODE>
static cudaError_t w8tc_mode(const CUtensorMap& mx, const W8TcArgs& a, int mp, cudaStream_t st) {
  if (mp == 16) return w8tc_launch_t<16, MODE>(mx, a, st);
  if (mp == 32) return w8tc_launch_t<32, MODE>(mx, a, st);
  if (mp == 48) return w8tc_launch_t<48, MODE>(mx, a, st);
  return w8tc_launch_t<64, MODE>(mx, a, st);
}

// K-split = cluster size (1..8): as many CTAs as fit two per SM in one wave,
// keeping at least two k64 steps per CTA.
int w8tc_pick_splits(int N, int K, int num_sms) {
  const int tiles = N / 128;
  int s = (2 * num_sms) / tiles;
  if (s > 8) s = 8;
  if (s > (K / 64) / 2) s = (K / 64) / 2;
  if (s < 1) s = 1;
  return s;
}

cudaError_t w8tc_launch(const int8_t* w_tiles, const W8Params& p, int mode, int* err, cudaStream_t st) {
  if (p.M < 1 || p.M > 64 || p.N % 128 || p.K % 64 || p.splits < 1 || p.splits > 8 ||
      p.K / 64 < p.splits)
    return cudaErrorInvalidValue;
  const int mp = (p.M + 15) / 16 * 16;
  if (reinterpret_cast<uintptr_t>(w_tiles) & 15) return cudaErrorInvalidValue;
  CUtensorMap mx;
  if (!map2d(&mx, p.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.K, p.M, 64, mp, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  W8TcArgs a{p, w_tiles, err};
  if (mode == kQKV) return w8tc_mode<kQKV>(mx, a, mp, st);
  if (mode == kResid) return w8tc_mode<kResid>(mx, a, mp, st);
  if (mode == kSiluMul) return w8tc_mode<kSiluMul>(mx, a, mp, st);
  if (mode == kStore) return w8tc_mode<kStore>(mx, a, mp, st);
  return cudaErrorInvalidValue;
}

cudaError_t w8_tilepack_launch(const int8_t* src, int n_src, int K, int8_t* dst, int grp, int gstride,
                               int base, cudaStream_t st) {
  if (K % 64) return cudaErrorInvalidValue;
  w8_tilepack_kernel<<<1024, 256, 0, st>>>(src, n_src, K, dst, grp, gstride, base);
  return cudaGetLastError();
}

}  // namespace dfl
