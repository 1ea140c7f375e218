// Dense context-side GEMMs on the 5th-gen tensor cores (tcgen05 + TMA).
//
//   D[M, N] = A[M, K] . B[N, K]^T      A, B K-major (row-major, K contiguous)
//
// Used for the two context projections of the draft forward whose M is the
// number of context rows (thousands):
//   * fc        (dflash.py:392):  target_hidden [rows, F*H] x Wfc [H, F*H]  (bf16)
//       epilogue: bf16 store + per-256-column partial sum of squares for the
//       following RMSNorm (hidden_norm).
//   * ctx K/V   (dflash.py:293-305): normalised context [rows, H] x the K|V
//       weights of all layers [L*2*NKV*128, H] (f16, exact int8 values; the
//       fp16 per-channel scale is applied in the epilogue).
//       epilogue: scale, per-head k RMSNorm + neox RoPE, f16 store into the
//       per-layer K / V buffers.
//
// Persistent: one CTA per SM walks output tiles 128 x 256 (blockIdx.x, +grid,
// ...) in a rasterised order (groups of 8 n-blocks, n fastest), so the tiles
// in flight at once share A and B rows in L2.  K step 64 (one 128-byte
// swizzle atom), 4-stage TMA ring across tile boundaries.  With more than
// 128 rows, clusters of two CTAs share 256 x 256 tiles instead
// (tcgen05.mma.cta_group::2, 6-stage rings of 32 KB: TcCfg below).
// Warp 0: TMA producer.  Warp 1: TMEM allocator + single-thread UMMA issuer
// (tcgen05.mma.cta_group::1.kind::f16, M=128 N=256 K=16) into one of two fp32
// accumulators (2 x 256 TMEM columns), so the epilogue of a tile overlaps the
// main loop of the next.  Warps 2-5: epilogue (tcgen05.ld, each thread owns one
// accumulator row, so per-row and per-head reductions are thread-local).
// Every mbarrier wait is bounded; a timeout sets the device error word and the
// CTA unwinds (TMEM is released on every path).
#include <algorithm>
#include <cstdlib>

#include "kernels.cuh"

namespace dfl {

constexpr int TC_BM = 128, TC_BN = 256, TC_BK = 64, TC_STAGES = 4;
constexpr int TC_A_BYTES = TC_BM * TC_BK * 2;   // 16 KB
constexpr int TC_B_BYTES = TC_BN * TC_BK * 2;   // 32 KB
constexpr int TC_THREADS = 192;
constexpr int TC_GROUP_N = 8;  // rasterisation: n-blocks per tile group

// PAIR: a cluster of two CTAs computes one 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256): each CTA stages its own 128 A rows and
// half of the 256 B rows, so a CTA's shared memory carries 32 KB per k-block
// instead of 48 KB, the ring gets 6 stages, and B crosses L2 once per pair.
template <bool PAIR>
struct TcCfg {
  static constexpr int NR = PAIR ? 2 : 1;                      // CTAs per tile
  static constexpr int STAGES = PAIR ? 6 : TC_STAGES;
  static constexpr int B_BYTES = TC_B_BYTES / NR;              // this CTA's B rows
  static constexpr int STAGE_BYTES = TC_A_BYTES + B_BYTES;
  static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024 + 256;
};

// tile t -> (m-block, n-block): groups of TC_GROUP_N n-blocks; inside a group
// the n-block runs fastest
__device__ __forceinline__ void tc_tile(int t, int nmb, int nnb, int& mb, int& nb) {
  const int g = t / (nmb * TC_GROUP_N);
  const int first = g * TC_GROUP_N;
  const int gw = min(TC_GROUP_N, nnb - first);
  const int r = t - g * nmb * TC_GROUP_N;
  mb = r / gw;
  nb = first + r % gw;
}



// Context K|V (per layer: K heads, then V heads, 128 columns each): tile
// column n-block nb runs over every layer's K blocks first and then every
// layer's V blocks, so a CTA's last tile is a V tile.  The last tile's
// epilogue overlaps nothing, and a V tile's (scale, store) takes ~8 us where a
// K tile's (RMSNorm, RoPE) takes ~24.  Identity when a layer's K half is not a
// whole number of 256-column blocks.
template <int MODE>
__device__ __forceinline__ int tc_nb_phys(int nb, int nnb, int nkv) {
  if (MODE != kTcCtxKV || nkv % 2) return nb;
  const int half = nkv / 2;          // 256-column blocks per K (or V) half of a layer
  const int kb = nnb / 2;            // all layers' K blocks
  const int v = nb >= kb ? 1 : 0;
  const int i = nb - v * kb;
  return (i / half) * (2 * half) + v * half + i % half;
}

// Work of CTA c (grid G, T tiles): tiles c, c + G, ... of the first
// R = T / G rounds; with a tail split S > 0 the T - R*G tiles of the last,
// partial round are cut along K into S parts each, P = (T - R*G) * S parts
// in all, and CTA c adds parts c, c + G, ... < P (part q: tail tile
// R*G + q / S, K part q % S).  With few tiles R is 0 and every tile is split.  A tail part writes its
// fp32 partial accumulator to the workspace; the last part of a tile to
// finish sums the parts in fixed order and runs the epilogue.
struct TcItem {
  int tile, kb0, kb1, part;   // part < 0: a whole tile
};
__device__ __forceinline__ TcItem tc_item(int ti, int T, int nk, int split, int G, int c) {
  const int R = T / G;
  if (split > 0 && ti >= R) {
    const int q = c + (ti - R) * G;
    const int part = q % split;
    return {R * G + q / split, part * nk / split, (part + 1) * nk / split, part};
  }
  return {c + ti * G, 0, nk, -1};
}
__device__ __forceinline__ int tc_items(int T, int split, int G, int c) {
  if (split > 0) {
    const int R = T / G;
    const int P = (T - R * G) * split;
    return R + (P > c ? (P - c + G - 1) / G : 0);
  }
  return T > c ? (T - c + G - 1) / G : 0;
}

// One 128-column head of this thread's accumulator row (TMEM columns tcol ..
// tcol+127): y = acc * scale, then, when nw is given, RMSNorm over the head
// (weight nw) and neox RoPE from the (cos, sin) table row cs; f16 store to
// dst.  Every lane of the warp calls it (tcgen05.ld is warp-wide); only rows
// with row_ok store.
__device__ __forceinline__ void tc_store_head(uint32_t tcol, const float* __restrict__ sc,
                                              const float* __restrict__ nw, const float2* __restrict__ cs,
                                              float eps, __half* dst, bool row_ok, float rowscale = 1.f) {
  float rstd = 1.f;
  if (nw) {
    float ss = 0.f;
#pragma unroll 1
    for (int ch = 0; ch < 4; ++ch) {
      uint32_t r[32];
      tmem_ld32(tcol + ch * 32, r);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float y = __uint_as_float(r[e]) * __ldg(sc + ch * 32 + e) * rowscale;
        ss += y * y;
      }
    }
    rstd = rsqrtf(ss / 128.0f + eps);
  }
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    uint32_t r1[32], r2[32];
    tmem_ld32(tcol + half * 32, r1);
    tmem_ld32(tcol + 64 + half * 32, r2);
    tmem_ld_wait();
    if (row_ok) {
      uint32_t o1[16], o2[16];
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float a[2], b[2];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int d = half * 32 + e + t;
          float y1 = __uint_as_float(r1[e + t]) * __ldg(sc + d) * rowscale;
          float y2 = __uint_as_float(r2[e + t]) * __ldg(sc + d + 64) * rowscale;
          if (nw) {
            y1 = y1 * rstd * __ldg(nw + d);
            y2 = y2 * rstd * __ldg(nw + d + 64);
            const float2 t2 = __ldg(cs + d);
            a[t] = y1 * t2.x - y2 * t2.y;
            b[t] = y1 * t2.y + y2 * t2.x;
          } else {
            a[t] = y1;
            b[t] = y2;
          }
        }
        o1[e / 2] = pack_f16x2(a[0], a[1]);
        o2[e / 2] = pack_f16x2(b[0], b[1]);
      }
      uint4* d1 = reinterpret_cast<uint4*>(dst + half * 32);
      uint4* d2 = reinterpret_cast<uint4*>(dst + 64 + half * 32);
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        d1[v] = make_uint4(o1[4 * v], o1[4 * v + 1], o1[4 * v + 2], o1[4 * v + 3]);
        d2[v] = make_uint4(o2[4 * v], o2[4 * v + 1], o2[4 * v + 2], o2[4 * v + 3]);
      }
    }
  }
}

// tensor maps of the A column blocks (one, or one per source array)
template <int NSRC>
struct TcAMaps {
  CUtensorMap m[NSRC];
};

template <int AB_FMT, int MODE, int NSRC, bool PAIR>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ TcAMaps<NSRC> maps_a, const __grid_constant__ CUtensorMap map_b,
                   const TcParams p) {
  using CF = TcCfg<PAIR>;
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + CF::STAGES * CF::STAGE_BYTES);
  uint64_t* empty = full + CF::STAGES;
  uint64_t* accf = empty + CF::STAGES;  // [2] accumulator ready
  uint64_t* acce = accf + 2;           // [2] accumulator drained by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* tail_flag = abort_flag + 1;   // this CTA's tail part is a tile's last

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = p.K / TC_BK;
  // pair mode: tiles of 256 rows, CTA `rank` of the cluster owns rows rank*128.. of each
  const uint32_t rank = PAIR ? cluster_ctarank() : 0;
  const int G = PAIR ? (int)gridDim.x / 2 : (int)gridDim.x;
  const int cidx = PAIR ? (int)blockIdx.x / 2 : (int)blockIdx.x;
  const int nmb = (p.M + TC_BM * CF::NR - 1) / (TC_BM * CF::NR), nnb = p.N / TC_BN;
  const int ntiles = nmb * nnb;
  const int my_tiles = tc_items(ntiles, p.split, G, cidx);

  if (threadIdx.x == 0) {
    for (int s = 0; s < CF::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4 * CF::NR);   // the epilogue warps of every CTA of the tile
    }
    *abort_flag = 0;
    fence_mbar_init();
    for (int f = 0; f < NSRC && f * p.a_cols < p.K; ++f) prefetch_tmap(&maps_a.m[f]);
    prefetch_tmap(&map_b);
  }
  if (PAIR) {
    // both CTAs' barriers exist before any CTA signals its peer's
    __syncthreads();
    cluster_arrive_release();
    cluster_wait_acquire();
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, 2 * TC_BN);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, 2 * TC_BN);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int ti = 0; ti < my_tiles && ok; ++ti) {
        const TcItem w = tc_item(ti, ntiles, nk, p.split, G, cidx);
        int mb, nb;
        tc_tile(w.tile, nmb, nnb, mb, nb);
        nb = tc_nb_phys<MODE>(nb, nnb, p.nkv);
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = it % CF::STAGES;
          const uint32_t ph = (it / CF::STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.err, abort_flag)) { ok = false; break; }
          uint8_t* sa = smem + s * CF::STAGE_BYTES;
          int col = kb * TC_BK, f = 0;
          if (NSRC > 1) {
            f = col / p.a_cols;
            col -= f * p.a_cols;
          }
          if (PAIR) {
            // both CTAs' copies complete on rank 0's full barrier, which
            // expects the bytes of the pair (an odd CTA's copy may land before
            // rank 0 arms the barrier: the transaction count is signed)
            const uint32_t fb = mapa_shared(&full[s], 0);
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * CF::STAGE_BYTES);
            tma_load_2d_pair(sa, &maps_a.m[f], fb, col, (mb * 2 + (int)rank) * TC_BM);
            if (MODE == kTcArgmax)
              tma_load_2d_pair(sa + TC_A_BYTES, &map_b, fb, 0, ((2 * nb + (int)rank) * nk + kb) * 128);
            else
              tma_load_2d_pair(sa + TC_A_BYTES, &map_b, fb, kb * TC_BK, nb * TC_BN + (int)rank * 128);
            continue;
          }
          mbar_arrive_expect_tx(&full[s], CF::STAGE_BYTES);
          tma_load_2d(sa, &maps_a.m[f], &full[s], col, mb * TC_BM);
          if (MODE == kTcArgmax) {
            // B = the lm_head's pre-swizzled vocabulary tiles: 16 KB blocks
            // [vt][kb][128 rows][128 B], two 128-row tiles per n-block
#pragma unroll
            for (int t = 0; t < 2; ++t)
              tma_load_2d(sa + TC_A_BYTES + t * (TC_B_BYTES / 2), &map_b, &full[s], 0,
                          ((2 * nb + t) * nk + kb) * 128);
          } else {
            tma_load_2d(sa + TC_A_BYTES, &map_b, &full[s], kb * TC_BK, nb * TC_BN);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {   // in a pair, the even CTA issues for both
      constexpr uint32_t idesc = umma_idesc_f16(TC_BM * CF::NR, TC_BN, AB_FMT);
      int it = 0;
      bool ok = true;
      for (int ti = 0; ti < my_tiles && ok; ++ti) {
        const int b = ti & 1;
        if (!mbar_wait(&acce[b], ((ti >> 1) & 1) ^ 1, p.err, abort_flag)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * TC_BN;
        const TcItem w = tc_item(ti, ntiles, nk, p.split, G, cidx);
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = it % CF::STAGES;
          const uint32_t ph = (it / CF::STAGES) & 1;
          if (!mbar_wait(&full[s], ph, p.err, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * CF::STAGE_BYTES);
          const uint64_t adesc = umma_desc_sw128(sa);
          const uint64_t bdesc = umma_desc_sw128(sa + TC_A_BYTES);
#pragma unroll
          for (int k = 0; k < TC_BK / 16; ++k) {
            // advance 16 elements (32 bytes) inside the swizzle atom: +2 in 16-byte units
            if (PAIR)
              umma_f16_pair(acc, adesc + 2 * k, bdesc + 2 * k, idesc, (kb != w.kb0 || k != 0));
            else
              umma_f16(acc, adesc + 2 * k, bdesc + 2 * k, idesc, (kb != w.kb0 || k != 0));
          }
          if (PAIR)
            umma_commit_pair(&empty[s]);   // frees the stage in both CTAs
          else
            umma_commit(&empty[s]);
        }
        if (PAIR)
          umma_commit_pair(&accf[b]);  // both halves of the tile are ready
        else
          umma_commit(&accf[b]);  // fires once every MMA of the tile has retired
      }
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane quadrant (warp % 4)
    const int q = warp & 3;
    const int row_local = q * 32 + lane;
    for (int ti = 0; ti < my_tiles; ++ti) {
      const int buf = ti & 1;
      const TcItem w = tc_item(ti, ntiles, nk, p.split, G, cidx);
      int mb, nb;
      tc_tile(w.tile, nmb, nnb, mb, nb);
      nb = tc_nb_phys<MODE>(nb, nnb, p.nkv);
      const int n0 = nb * TC_BN;
      const int row = (mb * CF::NR + (int)rank) * TC_BM + row_local;
      bool row_ok = row < p.M;
      int ci = -1;   // tail counter of this part's (slot, rank), -1 for a whole tile
      // No epilogue warp leaves the loop early: after a timeout (the abort
      // flag) the items are walked without work, so every named barrier of
      // the tail parts below is reached by all four warps.
      const bool live = mbar_wait(&accf[buf], (ti >> 1) & 1, p.err, abort_flag) && !*abort_flag;
      if (live) tc_fence_after();
      const uint32_t tbase = tmem + buf * TC_BN + ((uint32_t)(q * 32) << 16);
      bool run = live;
      if (w.part >= 0) {
        const int slot = w.tile - (ntiles / G) * G;
        // partial of (slot, part, rank): every CTA half of a pair keeps its own rows
        float* mine = p.tail_part + (((size_t)slot * p.split + w.part) * CF::NR + rank) * (TC_BM * TC_BN);
        if (live) {
#pragma unroll 1
          for (int ch = 0; ch < TC_BN / 32; ++ch) {
            uint32_t r[32];
            tmem_ld32(tbase + ch * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) mine[(size_t)(ch * 32 + e) * TC_BM + row_local] = __uint_as_float(r[e]);
          }
        }
        __threadfence();
        named_bar_sync(2, 128);
        // The tile's parts finish together (equal K slices), so each waits,
        // bounded, until all have written their partials and then merges
        // and finishes its 1/split of the rows, instead of the last to
        // arrive taking all 128.  The counter counts arrivals to split, then
        // departures to 2 split (every part counts, after an abort too); the
        // last departure resets it for the next launch.
        ci = slot * CF::NR + (int)rank;
        if (threadIdx.x == 64) {
          atomicAdd(p.tail_cnt + ci, 1);
          bool arrived = true;
          for (uint32_t i = 0; ld_acquire_gpu(p.tail_cnt + ci) < p.split; ++i) {
            if (i >= kSpinLimit || *abort_flag) {
              if (!*abort_flag) atomicExch(p.err, kDevMbarTimeout);
              *abort_flag = 1;
              arrived = false;
              break;
            }
            __nanosleep(32);
          }
          *tail_flag = arrived;
        }
        named_bar_sync(2, 128);
        const int r0 = w.part * TC_BM / p.split, r1 = (w.part + 1) * TC_BM / p.split;
        row_ok = row_ok && row_local >= r0 && row_local < r1;
        // a warp with none of the part's rows skips the merge and the epilogue
        run = live && *tail_flag != 0 && __any_sync(0xffffffffu, row_local >= r0 && row_local < r1);
        if (run) {
          // sum the parts in fixed order into the accumulator (all lanes of
          // the warp; only the part's rows are stored by the epilogue)
          __threadfence();
          const float* base = p.tail_part + ((size_t)slot * p.split * CF::NR + rank) * (TC_BM * TC_BN);
#pragma unroll 1
          for (int ch = 0; ch < TC_BN / 32; ++ch) {
            // 32 independent loads per part, so they are all in flight at once
            const float* col = base + (size_t)(ch * 32) * TC_BM + row_local;
            float a[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) a[e] = __ldcg(col + (size_t)e * TC_BM);
            for (int q2 = 1; q2 < p.split; ++q2) {
              const float* cq = col + (size_t)q2 * CF::NR * (TC_BM * TC_BN);
              float v[32];
#pragma unroll
              for (int e = 0; e < 32; ++e) v[e] = __ldcg(cq + (size_t)e * TC_BM);
#pragma unroll
              for (int e = 0; e < 32; ++e) a[e] += v[e];
            }
            uint32_t r[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(a[e]);
            tmem_st32(tbase + ch * 32, r);
          }
          tmem_st_wait();
        }
      }
      if (run) {
        if (MODE == kTcFc && p.out_b16) {
          // hidden_norm fused: bf16(fc * w) here, 1/rms per row in the context K|V GEMM
          float ss = 0.f;
#pragma unroll 1
          for (int ch = 0; ch < TC_BN / 32; ++ch) {
            uint32_t r[32];
            tmem_ld32(tbase + ch * 32, r);
            tmem_ld_wait();
            if (row_ok) {
              const float* w = p.colw + n0 + ch * 32;
              uint32_t o[16];
#pragma unroll
              for (int e = 0; e < 32; e += 2) {
                const float a = __uint_as_float(r[e]), b = __uint_as_float(r[e + 1]);
                ss += a * a + b * b;
                o[e / 2] = pack_bf16x2(a * __ldg(w + e), b * __ldg(w + e + 1));
              }
              uint4* dst = reinterpret_cast<uint4*>(p.out_b16 + (size_t)row * p.N + n0 + ch * 32);
#pragma unroll
              for (int v = 0; v < 4; ++v) dst[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
            }
          }
          if (row_ok) p.sumsq_part[(size_t)nb * p.M + row] = ss;
        } else if (MODE == kTcFc || MODE == kTcStoreF32) {
          float ss = 0.f;
#pragma unroll 1
          for (int ch = 0; ch < TC_BN / 32; ++ch) {
            uint32_t r[32];
            tmem_ld32(tbase + ch * 32, r);
            tmem_ld_wait();
            if (row_ok) {
              float4* dst = reinterpret_cast<float4*>(p.out_f32 + (size_t)row * p.N + n0 + ch * 32);
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                const float4 f = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                             __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
                if (MODE == kTcFc) ss += f.x * f.x + f.y * f.y + f.z * f.z + f.w * f.w;
                dst[v] = f;
              }
            }
          }
          if (MODE == kTcFc && row_ok) p.sumsq_part[(size_t)nb * p.M + row] = ss;
        } else if (MODE == kTcCtxKV) {  // two 128-wide heads per tile
          // sequence and slot of this packed context row (rows >= M are never stored)
          const int crow = row_ok ? row : 0;
          const int bi = kv_seq_of_ctx_row(p.kv.seq, p.kv.nseq, crow);
          const KvSeq sq = p.kv.seq[bi];
          const int slot = kv_slot(p.kv, sq.n0 + crow - sq.ctx_start, sq.rs_pre);
          const int per_layer = 2 * p.nkv * 128;
          float rowscale = 1.f;   // hidden_norm's 1/rms of this context row
          if (p.row_sumsq) {
            float ssr = 0.f;
            for (int q3 = 0; q3 < p.row_parts; ++q3) ssr += __ldg(p.row_sumsq + (size_t)q3 * p.M + crow);
            rowscale = rsqrtf(ssr / static_cast<float>(p.row_dim) + p.eps);
          }
#pragma unroll 1
          for (int hh = 0; hh < 2; ++hh) {
            const int col0 = n0 + hh * 128;
            const int layer = col0 / per_layer;
            const int within = col0 - layer * per_layer;
            const bool is_v = within >= p.nkv * 128;
            const int kvh = (within % (p.nkv * 128)) / 128;
            __half* dst = (is_v ? p.v_out : p.k_out) + (size_t)layer * p.layer_stride +
                          (((size_t)sq.cseq * p.nkv + kvh) * p.kv.slots + slot) * 128;
            tc_store_head(tbase + hh * 128, p.scale + col0, is_v ? nullptr : p.k_norm + layer * 128,
                          p.rope + (size_t)crow * 64, p.eps, dst, row_ok, rowscale);
          }
        } else if (MODE == kTcBlkQKV) {  // block rows: q | k | v heads, two per tile
          const int m = row_ok ? row : 0;
          const int bi = m / p.block, j = m - bi * p.block;
          const KvSeq sq = p.kv.seq[bi];
          const int lrow = sq.n0 + (p.kv.seq[bi + 1].ctx_start - sq.ctx_start) + j;
          const int slot = kv_slot(p.kv, lrow, sq.rs_pre);
#pragma unroll 1
          for (int hh = 0; hh < 2; ++hh) {
            const int col0 = n0 + hh * 128;
            const int head = col0 / 128;
            __half* dst;
            const float* nw;
            if (head < p.n_q_heads) {
              dst = p.q_out + (((size_t)bi * p.n_q_heads + head) * p.block + j) * 128;
              nw = p.q_norm;
            } else {
              const bool is_k = head < p.n_q_heads + p.nkv;
              const int kvh = head - p.n_q_heads - (is_k ? 0 : p.nkv);
              dst = (is_k ? p.k_out : p.v_out) + (((size_t)sq.cseq * p.nkv + kvh) * p.kv.slots + slot) * 128;
              nw = is_k ? p.k_norm : nullptr;
            }
            tc_store_head(tbase + hh * 128, p.scale + col0, nw, p.rope + (size_t)(p.rope_row0 + m) * 64,
                          p.eps, dst, row_ok);
          }
        } else if (MODE == kTcResid) {  // h += acc * scale, per-256-column sum of h^2
          float ss = 0.f;
#pragma unroll 1
          for (int ch = 0; ch < TC_BN / 32; ++ch) {
            uint32_t r[32];
            tmem_ld32(tbase + ch * 32, r);
            tmem_ld_wait();
            if (row_ok) {
              float4* hp = reinterpret_cast<float4*>(p.h + (size_t)row * p.N + n0 + ch * 32);
              const float4* sc = reinterpret_cast<const float4*>(p.scale + n0 + ch * 32);
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                const float4 s4 = __ldg(sc + v);
                float4 h4 = hp[v];
                h4.x += __uint_as_float(r[4 * v]) * s4.x;
                h4.y += __uint_as_float(r[4 * v + 1]) * s4.y;
                h4.z += __uint_as_float(r[4 * v + 2]) * s4.z;
                h4.w += __uint_as_float(r[4 * v + 3]) * s4.w;
                ss += h4.x * h4.x + h4.y * h4.y + h4.z * h4.z + h4.w * h4.w;
                hp[v] = h4;
              }
            }
          }
          if (row_ok) p.sumsq_part[(size_t)nb * p.M + row] = ss;
        } else if (MODE == kTcSilu) {  // 128 gate columns, then the 128 matching up columns
#pragma unroll 1
          for (int ch = 0; ch < 4; ++ch) {
            uint32_t rg[32], ru[32];
            tmem_ld32(tbase + ch * 32, rg);
            tmem_ld32(tbase + 128 + ch * 32, ru);
            tmem_ld_wait();
            if (row_ok) {
              const float* sg = p.scale + n0 + ch * 32;
              const float* su = sg + 128;
              uint32_t o[16];
#pragma unroll
              for (int e = 0; e < 32; e += 2) {
                float a[2];
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                  const float g = __uint_as_float(rg[e + t]) * __ldg(sg + e + t);
                  const float u = __uint_as_float(ru[e + t]) * __ldg(su + e + t);
                  a[t] = (g / (1.0f + expf(-g))) * u;
                }
                o[e / 2] = pack_f16x2(a[0], a[1]);
              }
              uint4* dst = reinterpret_cast<uint4*>(p.act + (size_t)row * (p.N / 2) + nb * 128 + ch * 32);
#pragma unroll
              for (int v = 0; v < 4; ++v) dst[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
            }
          }
        } else {  // kTcArgmax: first index of the row maximum over the tile's columns < V
          float best = -INFINITY;
          int bidx = 0x7fffffff;
#pragma unroll 1
          for (int ch = 0; ch < TC_BN / 32; ++ch) {
            uint32_t r[32];
            tmem_ld32(tbase + ch * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int col = n0 + ch * 32 + e;
              const float x = __uint_as_float(r[e]);
              if (col < p.V && x > best) {
                best = x;
                bidx = col;
              }
            }
          }
          if (row_ok) {
            p.best_val[(size_t)nb * p.M + row] = best;
            p.best_idx[(size_t)nb * p.M + row] = bidx;
          }
        }
      }
      if (ci >= 0 && threadIdx.x == 64 && atomicAdd(p.tail_cnt + ci, 1) == 2 * p.split - 1)
        p.tail_cnt[ci] = 0;   // every part of the tile is done
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {  // accumulator free for tile ti + 2 (rank 0 issues the MMAs of a pair)
        if (PAIR)
          mbar_arrive_cluster(mapa_shared(&acce[buf], 0));
        else
          mbar_arrive(&acce[buf]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) {
    // no CTA of the pair leaves while its peer may still signal its barriers
    // or the tensor core may still read its shared memory
    cluster_arrive_release();
    cluster_wait_acquire();
  }
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem, 2 * TC_BN);
    else
      tmem_dealloc(tmem, 2 * TC_BN);
  }
}

// ------------------------------------------------------------------ host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 2-D K-major map: inner dim `inner` (elements), outer dim rows `ld` elements
// apart; box 64 x box_rows, 128B swizzle (or none, for data stored pre-swizzled)
static bool make_map(CUtensorMap* map, const void* base, bool bf16, uint64_t inner, uint64_t rows,
                     uint32_t box_rows, uint64_t ld, bool swizzle = true) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  if (!base || (reinterpret_cast<uintptr_t>(base) & 15) || (ld * 2) % 16 || ld < inner) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {TC_BK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// CTA pairs are on unless DFLASH_TC_PAIRS=0 (read once), which keeps the
// single-CTA kernel for comparison runs
static bool tc_pairs_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("DFLASH_TC_PAIRS");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// Tail split: the tiles of the partial last round (all tiles when there are
// fewer than SMs) are cut along K into S parts spread over the grid.  S
// minimises the makespan in tile units, R + ceil(tail * S / G) * (1 / S + c),
// where c, the cost of writing and merging a partial accumulator, is taken
// as 10 k-blocks of MMA; each part has at least 4 k-blocks and the parts fit
// cap_parts partial slots.  0 (no split) when the tiles fill whole rounds or
// no S >= 2 saves at least 5%.  Returns S and the grid to launch.
int tc_tail_split(int tiles, int sms, int nk, int cap_parts, int* grid_out) {
  int grid = tiles < sms ? tiles : sms;
  *grid_out = grid;
  if (cap_parts <= 0 || sms < 1) return 0;
  const int R = tiles / sms, tail = tiles - R * sms;
  if (tail == 0) return 0;
  const double whole = R + 1.0, c = 10.0 / nk;
  double best = whole;
  int bs = 0;
  for (int s = 2; s <= nk / 4 && (long long)tail * s <= cap_parts; ++s) {
    const double m = R + (double)((tail * s + sms - 1) / sms) * (1.0 / s + c);
    if (m < best - 1e-9) {
      best = m;
      bs = s;
    }
  }
  if (bs == 0 || best > 0.95 * whole) return 0;
  // with full rounds the grid is every SM; otherwise as many CTAs as parts, up to the SMs
  *grid_out = R > 0 ? sms : (tail * bs < sms ? tail * bs : sms);
  return bs;
}

// clusters of two CTAs of `kern` that fit on the device at once (an SM without
// a partner in its GPC cannot host half a pair); cached per instantiation
template <class Kern>
static int tc_max_pairs(Kern kern, size_t smem, int* cache) {
  if (*cache >= 0) return *cache;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
  *cache = n;
  return n;
}

template <int FMT, int MODE, int NSRC, bool PAIR>
static cudaError_t tc_launch_t(const TcAMaps<NSRC>& ma, const CUtensorMap& mb, TcParams p, cudaStream_t st) {
  using CF = TcCfg<PAIR>;
  auto kern = tc_gemm_kernel<FMT, MODE, NSRC, PAIR>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)CF::SMEM);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  DFL_TRY(cudaGetDevice(&dev));
  DFL_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  DFL_TRY(max_smem_carveout(kern));
  int units = sms;   // CTAs, or CTA pairs, resident at once
  if (PAIR) {
    static int cache = -1;
    units = std::min(sms / 2, tc_max_pairs(kern, CF::SMEM, &cache));
    if (units < 1) return cudaErrorInvalidConfiguration;
  }
  const int tiles = (p.N / TC_BN) * ((p.M + TC_BM * CF::NR - 1) / (TC_BM * CF::NR));
  const bool ws = p.tail_part != nullptr && p.tail_cnt != nullptr;
  int grid = 0;
  p.split = tc_tail_split(tiles, units, p.K / TC_BK, ws ? p.tail_cap / CF::NR : 0, &grid);
  if (PAIR)
    return launch_pdl_cluster_smem(kern, dim3(2 * grid), dim3(TC_THREADS), 2, CF::SMEM, st, ma, mb, p);
  return launch_pdl(kern, dim3(grid), dim3(TC_THREADS), CF::SMEM, st, ma, mb, p);
}

template <int FMT, int MODE, int NSRC>
static cudaError_t tc_launch_pick(const TcAMaps<NSRC>& ma, const CUtensorMap& mb, const TcParams& p, bool pair,
                                  cudaStream_t st) {
  return pair ? tc_launch_t<FMT, MODE, NSRC, true>(ma, mb, p, st) : tc_launch_t<FMT, MODE, NSRC, false>(ma, mb, p, st);
}

template <int NSRC>
static cudaError_t tc_dispatch(const TcAMaps<NSRC>& ma, const CUtensorMap& mb, bool bf16, int mode,
                               const TcParams& p, bool pair, cudaStream_t st) {
  if (bf16) {
    if (mode == kTcFc) return tc_launch_pick<1, kTcFc, NSRC>(ma, mb, p, pair, st);
    if (mode == kTcStoreF32) return tc_launch_pick<1, kTcStoreF32, NSRC>(ma, mb, p, pair, st);
    if constexpr (NSRC == 1) {
      if (mode == kTcArgmax) return tc_launch_pick<1, kTcArgmax, 1>(ma, mb, p, pair, st);
      if (mode == kTcCtxKV) return tc_launch_pick<1, kTcCtxKV, 1>(ma, mb, p, pair, st);
    }
  } else {
    if constexpr (NSRC == 1) {
      if (mode == kTcCtxKV) return tc_launch_pick<0, kTcCtxKV, 1>(ma, mb, p, pair, st);
      if (mode == kTcBlkQKV) return tc_launch_pick<0, kTcBlkQKV, 1>(ma, mb, p, pair, st);
      if (mode == kTcResid) return tc_launch_pick<0, kTcResid, 1>(ma, mb, p, pair, st);
      if (mode == kTcSilu) return tc_launch_pick<0, kTcSilu, 1>(ma, mb, p, pair, st);
    }
    if (mode == kTcStoreF32) return tc_launch_pick<0, kTcStoreF32, NSRC>(ma, mb, p, pair, st);
  }
  return cudaErrorInvalidValue;
}

// A [M, K] and B [N, K] K-major, both bf16 or both f16.  mode: TcMode.  For
// kTcArgmax, B is the lm_pack tile array of a vocabulary of p.V rows and N is
// p.V rounded up to 256.
cudaError_t tc_gemm_launch_src(const TcSources& a, const void* B, bool bf16, int mode, TcParams p,
                               cudaStream_t st) {
  if (p.M < 1 || p.N % TC_BN || p.K % TC_BK || p.K < TC_BK) return cudaErrorInvalidValue;
  if (a.n < 1 || a.n > kTcMaxSrc || a.cols < TC_BK || a.cols % TC_BK || (long long)a.n * a.cols != p.K)
    return cudaErrorInvalidValue;
  p.a_cols = a.cols;
  // CTA pairs (M = 256 tiles) once there are two 128-row blocks to share B
  const bool pair = p.M > TC_BM && tc_pairs_enabled();
  CUtensorMap mb;
  if (mode == kTcArgmax) {
    const uint64_t vt = ((uint64_t)p.V + 127) / 128;
    if (!bf16 || p.V < 1 || (uint64_t)p.N < vt * 128 || (uint64_t)p.N > vt * 128 + 128) return cudaErrorInvalidValue;
    if (!make_map(&mb, B, true, TC_BK, vt * (p.K / TC_BK) * 128, 128, TC_BK, false)) return cudaErrorInvalidValue;
  } else if (!make_map(&mb, B, bf16, p.K, p.N, pair ? TC_BN / 2 : TC_BN, p.K)) {
    return cudaErrorInvalidValue;
  }
  if (a.n == 1) {
    TcAMaps<1> ma;
    if (!make_map(&ma.m[0], a.ptr[0], bf16, a.cols, p.M, TC_BM, a.ld[0])) return cudaErrorInvalidValue;
    return tc_dispatch<1>(ma, mb, bf16, mode, p, pair, st);
  }
  if (mode != kTcFc && mode != kTcStoreF32) return cudaErrorInvalidValue;
  TcAMaps<kTcMaxSrc> ma;
  for (int f = 0; f < a.n; ++f)
    if (!make_map(&ma.m[f], a.ptr[f], bf16, a.cols, p.M, TC_BM, a.ld[f])) return cudaErrorInvalidValue;
  for (int f = a.n; f < kTcMaxSrc; ++f) ma.m[f] = ma.m[0];
  return tc_dispatch<kTcMaxSrc>(ma, mb, bf16, mode, p, pair, st);
}

cudaError_t tc_gemm_launch(const void* A, const void* B, bool bf16, int mode, const TcParams& p,
                           cudaStream_t st) {
  TcSources a{};
  a.ptr[0] = A;
  a.ld[0] = p.K;
  a.n = 1;
  a.cols = p.K;
  return tc_gemm_launch_src(a, B, bf16, mode, p, st);
}

}  // namespace dfl
