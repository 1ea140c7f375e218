// W8A16 skinny GEMM on the 5th-gen tensor cores (tcgen05 + TMA), for the
// block rows of the draft forward (q|k|v, o, gate|up, down projections).
//
//   Y[m, n] = scale[n] * sum_k X[m, k] * Wq[n, k]      m < M <= 64, Wq int8
//
// Swap-AB: the 128 output channels of a tile are the UMMA M dimension and the
// (padded) activation rows are N (16..64), so one tcgen05.mma.kind::f16
// M=128 N=MP K=16 covers a whole tile.
//
// Persistent, one CTA per SM.  CTAs form groups of S (the K-split); group g
// walks tiles g, g + groups, ... and CTA `split` of the group covers the same
// K-slice of each of them, so every CTA streams the same number of bytes.
// Roles (14 warps):
//   warp 0     producer: each tile's k64 weight block is one contiguous 8 KB
//              run of the packed weights (cp.async.bulk); the f16 activation
//              tile [MP x 64] arrives by TMA with the 128-byte swizzle.  A deep
//              ring (NA stages) keeps ~100 KB of weights in flight per SM.
//   warps 2-9  converters: int8 -> 128-byte-swizzled f16 tile in a 4-stage
//              ring (PRMT with 0x6464 builds 1024+u, one f16x2 subtract
//              recovers q exactly), fence.proxy.async, arrive.
//   warp 1     single-thread UMMA issue into one of two 128 x MP fp32 TMEM
//              accumulators; tcgen05.commit frees the ring slots.
//   warps 10-13 epilogue of the previous tile while the next one streams: with
//              S > 1 each CTA writes its fp32 partial to global scratch and
//              the last CTA of the tile (per-tile arrival counter) sums the S
//              partials in split order (deterministic) and runs the fused
//              epilogue of kernels.cuh (kStore / kQKV / kResid / kSiluMul).
// The fp16 per-channel scale is applied in the epilogue (int8 values are exact
// in f16, so the product is the reference's q * s up to fp32 rounding).
// Every mbarrier wait is bounded; a timeout raises the device error word and
// the CTA unwinds (TMEM released on every path).
#include "kernels.cuh"

namespace dfl {

constexpr int WP_THREADS = 448;  // 14 warps: producer, MMA, 8 converters, 4 epilogue
constexpr int WP_NCW = 8;        // converter warps
constexpr int WP_NB = 4;         // converted f16 ring
constexpr int WP_W8 = 128 * 64;  // int8 tile bytes per k64
constexpr int WP_WF = 128 * 128; // f16 tile bytes per k64
constexpr int WP_SMEM_BUDGET = 206 * 1024;

template <int MP>
struct WpCfg {
  static constexpr int X_BYTES = MP * 128;
  static constexpr int A_STAGE = X_BYTES + WP_W8;  // [X swizzled | int8 weights]
  static constexpr int RED_BYTES = MP * 129 * 4;  // S == 1 epilogue staging [MP][129]
  static constexpr int NA_RAW = (WP_SMEM_BUDGET - WP_NB * WP_WF - RED_BYTES) / A_STAGE;
  static constexpr int NA = NA_RAW > 16 ? 16 : NA_RAW;
  static constexpr int RING_BYTES = WP_NB * WP_WF + NA * A_STAGE;
  static constexpr uint32_t ACC_COLS = MP <= 32 ? 32 : 64;
  static constexpr size_t SMEM = (size_t)RING_BYTES + RED_BYTES + 1024 + 512;
};

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
__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
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

struct WpArgs {
  W8Params p;
  const int8_t* w_tiles;  // [N/128][K/64][128 rows][64 B]
  float* part;            // [tiles][S][MP][128] fp32 split partials (S > 1)
  int* counters;          // [tiles] arrival counters, zero between launches
  int groups;             // grid = groups * S
  int* err;
};

// Fused epilogue for one activation row m of tile `tile` (a warp; lane owns
// EPC consecutive channels).  v / u hold the unscaled sums.
template <int MODE>
__device__ __forceinline__ void w8_epilogue_row(const W8Params& p, int tile, int m, int lane,
                                                float (&v)[4], float (&u)[4]) {
  constexpr int EPC = (MODE == kSiluMul) ? 2 : 4;
  const int gch = tile * 128 + lane * EPC;
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
    *reinterpret_cast<uint32_t*>(p.act + (size_t)m * (p.N / 2) + tile * 64 + lane * 2) = pack_f16x2(o[0], o[1]);
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
      rope_lane_t(v, lane, p.rope + (size_t)(p.rope_blk0 + m) * 64);
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
      const int lrow = p.kv.n0[bi] + (p.kv.ctx_start[bi + 1] - p.kv.ctx_start[bi]) + j;
      const int slot = kv_slot(p.kv, lrow, p.kv.rs_pre[bi]);
      dstp = base + (((size_t)bi * p.n_kv_heads + kvh) * p.kv.slots + slot) * 128;
    }
    *reinterpret_cast<uint2*>(dstp + lane * 4) = o;
  }
}

template <int MP, int MODE>
__global__ void __launch_bounds__(WP_THREADS, 1)
    w8p_kernel(const __grid_constant__ CUtensorMap map_x, const WpArgs args) {
  using C = WpCfg<MP>;
  const W8Params& p = args.p;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ringB = smem;                       // [NB][128 x 128 B] swizzled f16 weights
  uint8_t* ringA = smem + WP_NB * WP_WF;       // [NA][X | int8]
  float* red = reinterpret_cast<float*>(smem + C::RING_BYTES);  // [MP][129], S == 1 only
  uint64_t* fullA = reinterpret_cast<uint64_t*>(smem + C::RING_BYTES + C::RED_BYTES);
  uint64_t* emptyA = fullA + C::NA;
  uint64_t* convd = emptyA + C::NA;
  uint64_t* freeB = convd + WP_NB;
  uint64_t* accf = freeB + WP_NB;  // [2]
  uint64_t* acce = accf + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int S = p.splits;
  const int group = blockIdx.x / S;
  const int split = blockIdx.x % S;
  const int tiles = p.N / 128;
  const int ntile = tiles > group ? (tiles - group + args.groups - 1) / args.groups : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb_all = p.K / 64;
  const int kb0 = split * nkb_all / S;
  const int nkb = (split + 1) * nkb_all / S - kb0;
  const int total = ntile * nkb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NA; ++s) {
      mbar_init(&fullA[s], 1);
      mbar_init(&emptyA[s], 1);
    }
    for (int s = 0; s < WP_NB; ++s) {
      mbar_init(&convd[s], WP_NCW);
      mbar_init(&freeB[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&map_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * C::ACC_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int it = 0; it < total; ++it) {
        const int ti = it / nkb, kb = it - ti * nkb;
        const int tile = group + ti * args.groups;
        const int s = it % C::NA;
        if (!mbar_wait(&emptyA[s], ((it / C::NA) & 1) ^ 1, args.err, abort_flag)) break;
        uint8_t* st = ringA + s * C::A_STAGE;
        mbar_arrive_expect_tx(&fullA[s], C::A_STAGE);
        bulk_load(st + C::X_BYTES, args.w_tiles + ((size_t)tile * nkb_all + kb0 + kb) * WP_W8, WP_W8,
                  &fullA[s]);
        tma_load_2d(st, &map_x, &fullA[s], (kb0 + kb) * 64, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(128, MP, 0);
      int it = 0;
      bool ok = true;
      for (int ti = 0; ti < ntile && ok; ++ti) {
        const int b = ti & 1;
        if (!mbar_wait(&acce[b], ((ti >> 1) & 1) ^ 1, args.err, abort_flag)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * C::ACC_COLS;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int sa = it % C::NA, sb = it % WP_NB;
          if (!mbar_wait(&convd[sb], (it / WP_NB) & 1, args.err, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = umma_desc_sw128(smem_u32(ringB + sb * WP_WF));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(ringA + sa * C::A_STAGE));
#pragma unroll
          for (int k = 0; k < 4; ++k) umma_f16(acc, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0);
          umma_commit(&emptyA[sa]);
          umma_commit(&freeB[sb]);
        }
        umma_commit(&accf[b]);
      }
    }
  } else if (warp < 2 + WP_NCW) {
    // converters: piece c = 128*i + t is 16 int8 of row c/4, k 16*(c%4) .. +15;
    // reads are consecutive 16-byte pieces and the two 16-byte f16 writes of a
    // quarter-warp land on 8 distinct swizzled slots: no bank conflicts.
    const int t = threadIdx.x - 64;  // 0 .. 32*NCW-1
    for (int it = 0; it < total; ++it) {
      const int sa = it % C::NA, sb = it % WP_NB;
      if (!mbar_wait(&fullA[sa], (it / C::NA) & 1, args.err, abort_flag)) break;
      if (!mbar_wait(&freeB[sb], ((it / WP_NB) & 1) ^ 1, args.err, abort_flag)) break;
      const uint32_t src = smem_u32(ringA + sa * C::A_STAGE + C::X_BYTES);
      const uint32_t dstb = smem_u32(ringB + sb * WP_WF);
#pragma unroll
      for (int i = 0; i < 512 / (32 * WP_NCW); ++i) {
        const int c = i * 32 * WP_NCW + t;
        const int r = c >> 2, ch = c & 3;
        uint4 lo, hi;
        i8x16_to_f16x16(lds128_u(src + c * 16), lo, hi);
        const uint32_t dst = dstb + r * 128;
        sts128_u(dst + (((2 * ch) ^ (r & 7)) << 4), lo);
        sts128_u(dst + (((2 * ch + 1) ^ (r & 7)) << 4), hi);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&convd[sb]);
    }
  } else {
    // epilogue warps -> TMEM lane quadrant warp % 4 (= channels q*32 ..)
    const int q = warp & 3;
    const int et = threadIdx.x - 32 * (2 + WP_NCW);  // 0..127
    constexpr int EPC = (MODE == kSiluMul) ? 2 : 4;
    for (int ti = 0; ti < ntile; ++ti) {
      const int b = ti & 1;
      const int tile = group + ti * args.groups;
      if (!mbar_wait(&accf[b], (ti >> 1) & 1, args.err, abort_flag)) break;
      tc_fence_after();
      uint32_t r[MP];
#pragma unroll
      for (int c0 = 0; c0 < MP; c0 += 32) {
        uint32_t rr[32];
        tmem_ld32(tmem + b * C::ACC_COLS + ((uint32_t)(q * 32) << 16) + c0, rr);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (c0 + e < MP) r[c0 + e] = rr[e];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[b]);  // accumulator free for tile ti + 2
      const int ch = q * 32 + lane;
      if (S == 1) {
        // own tile: stage the accumulator in shared memory rows and run the epilogue
#pragma unroll
        for (int m = 0; m < MP; ++m) red[m * 129 + ch] = __uint_as_float(r[m]);
        named_bar(1, 128);
        for (int m = q; m < p.M; m += 4) {
          float v[4], u[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            v[e] = (e < EPC) ? red[m * 129 + lane * EPC + e] : 0.f;
            u[e] = (MODE == kSiluMul && e < EPC) ? red[m * 129 + 64 + lane * EPC + e] : 0.f;
          }
          w8_epilogue_row<MODE>(p, tile, m, lane, v, u);
        }
        named_bar(1, 128);
      } else {
        // split partial -> global [tile][split][m][128], coalesced per row
        float* dst = args.part + ((size_t)tile * S + split) * MP * 128;
#pragma unroll
        for (int m = 0; m < MP; ++m) dst[m * 128 + ch] = __uint_as_float(r[m]);
        __threadfence();
        named_bar(1, 128);
        if (et == 0) *last_flag = (atomicAdd(args.counters + tile, 1) == S - 1);
        named_bar(1, 128);
        if (*last_flag) {
          __threadfence();
          const float* src = args.part + (size_t)tile * S * MP * 128;
          // two rows per pass, every split's partial loaded before any add
          for (int m0 = q; m0 < p.M; m0 += 8) {
            float4 va[2][8], ua[2][8];
#pragma unroll
            for (int rr = 0; rr < 2; ++rr)
#pragma unroll
              for (int s = 0; s < 8; ++s) {
                const int m = m0 + 4 * rr;
                va[rr][s] = make_float4(0.f, 0.f, 0.f, 0.f);
                ua[rr][s] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (s < S && m < p.M) {
                  const float* rowp = src + ((size_t)s * MP + m) * 128;
                  if (EPC == 4) {
                    va[rr][s] = __ldcg(reinterpret_cast<const float4*>(rowp + lane * 4));
                  } else {
                    const float2 g2 = __ldcg(reinterpret_cast<const float2*>(rowp + lane * 2));
                    const float2 u2 = __ldcg(reinterpret_cast<const float2*>(rowp + 64 + lane * 2));
                    va[rr][s] = make_float4(g2.x, g2.y, 0.f, 0.f);
                    ua[rr][s] = make_float4(u2.x, u2.y, 0.f, 0.f);
                  }
                }
              }
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
              const int m = m0 + 4 * rr;
              if (m < p.M) {
                float v[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int s = 0; s < 8; ++s) {  // fixed split order: deterministic
                  v[0] += va[rr][s].x; v[1] += va[rr][s].y; v[2] += va[rr][s].z; v[3] += va[rr][s].w;
                  u[0] += ua[rr][s].x; u[1] += ua[rr][s].y;
                }
                w8_epilogue_row<MODE>(p, tile, m, lane, v, u);
              }
            }
          }
          if (et == 0) args.counters[tile] = 0;  // ready for the next launch
        }
        named_bar(1, 128);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * C::ACC_COLS);
  }
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

static bool map_f16_rows(CUtensorMap* m, const void* base, uint64_t K, uint64_t rows, uint32_t box_rows) {
  EncodeTiledFn2 enc = encode_fn();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15) || (K * 2) % 16) return false;
  cuuint64_t dims[2] = {K, rows};
  cuuint64_t strides[1] = {K * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// K-split S in 1..8 and groups = floor(SMs / S) from a small cost model:
// a tile slice streams nkb/S blocks of 8 KB at ~45 GB/s per SM; with S > 1
// every tile also pays a split-K merge (~4 us, hidden behind the next tile's
// stream when that is longer, exposed once at the end).
void w8tc_plan(int N, int K, int num_sms, int* splits, int* groups) {
  const int tiles = N / 128, nkb = K / 64;
  const double t_kb = 8192.0 / 45e3;  // us per k64 block per SM
  double best = 1e30;
  int bs = 1, bg = num_sms < tiles ? num_sms : tiles;
  for (int s = 1; s <= 8 && s <= nkb / 2; ++s) {
    int g = num_sms / s;
    if (g > tiles) g = tiles;
    if (g < 1) break;
    const int per = (tiles + g - 1) / g;
    const double epi = s > 1 ? 4.0 : 1.0;
    const double slice = (double)nkb / s * t_kb;
    const double est = per * (slice > epi ? slice : epi) + epi;
    if (est < best - 1e-9) { best = est; bs = s; bg = g; }
  }
  *splits = bs;
  *groups = bg;
}

size_t w8tc_part_floats(int N, int K, int M, int num_sms) {
  int s, g;
  w8tc_plan(N, K, num_sms, &s, &g);
  const int mp = (M + 15) / 16 * 16;
  return s > 1 ? (size_t)(N / 128) * s * mp * 128 : 0;
}

template <int MP, int MODE>
static cudaError_t w8p_launch_t(const CUtensorMap& mx, const WpArgs& a, cudaStream_t st) {
  using C = WpCfg<MP>;
  const size_t smem = C::SMEM;
  auto kern = w8p_kernel<MP, MODE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<a.groups * a.p.splits, WP_THREADS, smem, st>>>(mx, a);
  return cudaGetLastError();
}

template <int MODE>
static cudaError_t w8p_mode(const CUtensorMap& mx, const WpArgs& a, int mp, cudaStream_t st) {
  if (mp == 16) return w8p_launch_t<16, MODE>(mx, a, st);
  if (mp == 32) return w8p_launch_t<32, MODE>(mx, a, st);
  if (mp == 48) return w8p_launch_t<48, MODE>(mx, a, st);
  return w8p_launch_t<64, MODE>(mx, a, st);
}

cudaError_t w8tc_launch(const int8_t* w_tiles, const W8Params& pin, int mode, int* err, float* part,
                        size_t part_floats, int* counters, int num_sms, cudaStream_t st) {
  if (pin.M < 1 || pin.M > 64 || pin.N % 128 || pin.K % 128) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(w_tiles) & 15) return cudaErrorInvalidValue;
  W8Params p = pin;
  int groups = 1;
  w8tc_plan(p.N, p.K, num_sms, &p.splits, &groups);
  const int mp = (p.M + 15) / 16 * 16;
  if (p.splits > 1 && (!part || !counters || part_floats < (size_t)(p.N / 128) * p.splits * mp * 128))
    return cudaErrorInvalidValue;
  CUtensorMap mx;
  if (!map_f16_rows(&mx, p.x, p.K, p.M, mp)) return cudaErrorInvalidValue;
  WpArgs a{p, w_tiles, part, counters, groups, err};
  if (mode == kQKV) return w8p_mode<kQKV>(mx, a, mp, st);
  if (mode == kResid) return w8p_mode<kResid>(mx, a, mp, st);
  if (mode == kSiluMul) return w8p_mode<kSiluMul>(mx, a, mp, st);
  if (mode == kStore) return w8p_mode<kStore>(mx, a, mp, st);
  return cudaErrorInvalidValue;
}

cudaError_t w8_tilepack_launch(const int8_t* src, int n_src, int K, int8_t* dst, int grp, int gstride,
                               int base, cudaStream_t st) {
  if (K % 64) return cudaErrorInvalidValue;
  w8_tilepack_kernel<<<1024, 256, 0, st>>>(src, n_src, K, dst, grp, gstride, base);
  return cudaGetLastError();
}

}  // namespace dfl
