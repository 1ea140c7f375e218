// W8A16 skinny GEMM on the 5th-gen tensor cores for the block rows of the
// draft forward (q|k|v, o, gate|up, down projections).
//
//   Y[m, n] = scale[n] * sum_k X[m, k] * Wq[n, k]      m < M <= 64, Wq int8
//
// The activations run on the int8 tensor pipe (tcgen05.mma kind::i8) as
// three int8 limbs.  Each row m gets a power-of-two scale 2^(e_m - 20),
// where 2^e_m bounds max|x|.  Then x * 2^(20 - e_m) rounds to an integer
// q, |q| < 2^20, written as q = l0 + 128 l1 + 16384 l2 with
// l0, l1 in [-64, 63] and l2 in [-64, 64].
// The rows come as fp32 (the normed residual rows and silu(g) * u) or as f16
// (the attention output of a single-split step, a convex combination of f16 V
// rows): no f16 range limit applies before the split.  Every element keeps an
// absolute error of at most 2^(e_m - 21): 20 significant bits at the row
// maximum, and an f16 input within 2^10 of it is exact.  The weight-limb products accumulate
// exactly in int32 (|sum| < 127 * 64 * K < 2^31 for K <= 2^18).  Hence the
// integer sums, recombined in fp32 and scaled, are the W8A16 product with no
// rounding inside the dot product.
//
// Why: weights go straight from the bulk-copy ring into the MMA, as the
// lm_head kernel does.  No int8 -> f16 conversion pass through shared memory
// remains, which was the bound of the f16 formulation.
//
// Swap-AB: the 128 output channels of a tile are UMMA M.  The 3 * MP limb rows
// (MP = M padded to 16) are N.  One k128 block of a tile is
// 4 x tcgen05.mma.kind::i8 M=128 N=3MP K=32.
//
// Persistent, one CTA per SM, 6 warps.  A CTA works through "segments":
// k-block ranges of one 128-channel tile accumulated into one TMEM buffer.
// Two schedules share the kernel:
//   split    CTAs form groups of S.  Group g takes tiles g, g + groups, ...;
//            CTA `split` of the group takes the same K-slice of each of them.
//   stream-K the U = tiles * K/128 (tile, k-block) units, tile-major, are cut
//            into G equal contiguous runs, one per CTA.  A run covers whole
//            tiles and at most two partial ones.
// The host picks stream-K for long K (>= 64 k-blocks), where a split plan
// leaves many partial tiles to merge at the end, and the split plan otherwise
// (it was faster on the 40-block shapes of the 27B draft).
//   warp 0   producer: the tile's k128 weight block, 16 KB, is one contiguous
//            pre-swizzled run (cp.async.bulk); the limb tile [3MP x 128 B]
//            arrives by TMA with the 128-byte swizzle.
//   warp 1   single-thread UMMA issue into one of two int32 TMEM accumulators;
//            tcgen05.commit frees ring stages.
//   warps 2-5 epilogue of the previous segment while the next one streams.  A
//            segment that is a whole tile goes straight to the fused
//            epilogue.  Otherwise the CTA writes its fp32 partial to the
//            tile's slot in global scratch; the last of the tile's CTAs
//            (per-tile arrival counter) sums the partials in slot order
//            (deterministic) and runs the fused epilogue:
//     kStore   : Y as f16
//     kQKV     : per-head RMSNorm + neox RoPE for q and k heads, plain v,
//                written into the KvMap K/V layout (dflash.py:290-305)
//     kResid   : h += Y (fp32 residual stream) and per-128-channel sum of h^2
//                partials for the next RMSNorm (dflash.py:356, :361)
//     kSiluMul : each 128-channel tile holds 64 gate and the 64 matching up
//                channels -> silu(g) * u (dflash.py:330)
// Every mbarrier wait is bounded; a timeout raises the device error word and
// the CTA unwinds (TMEM released on every path).
#include <algorithm>

#include "kernels.cuh"

namespace dfl {

constexpr int WI_THREADS = 192;       // producer, MMA, 4 epilogue warps
constexpr int WI_WB = 128 * 128;      // int8 weight block: 128 channels x k128
constexpr int WI_SMEM_BUDGET = 200 * 1024;

template <int MP>
struct WiCfg {
  static constexpr int NB = 3 * MP;                // UMMA N: three limbs of MP rows
  static constexpr int X_BYTES = NB * 128;         // limb tile per k128
  static constexpr int STAGE = WI_WB + X_BYTES;    // multiple of 1024
  static constexpr int RED_BYTES = MP * 129 * 4;   // S == 1 epilogue staging [MP][129]
  static constexpr int NS_RAW = (WI_SMEM_BUDGET - RED_BYTES) / STAGE;
  static constexpr int NS = NS_RAW > 12 ? 12 : NS_RAW;
  static constexpr uint32_t ACC_COLS = NB <= 64 ? 64 : (NB <= 128 ? 128 : 256);
  static constexpr size_t SMEM = (size_t)NS * STAGE + RED_BYTES + 1024 + 256;
};

__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// kind::i8 instruction descriptor: s32 accumulate, signed int8 A and B, K-major
__host__ __device__ constexpr uint32_t umma_idesc_s8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
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

struct WiArgs {
  W8Params p;
  const int8_t* w_tiles;  // [N/128][K/128][128 rows][128 B], 16-byte chunks swizzled
  float* part;            // [tiles][maxseg][MP][128] fp32 partials of split tiles
  int* counters;          // [tiles] arrival counters, zero between launches
  int maxseg;             // partial slots per tile (<= 8)
  int stream_k;           // 1: stream-K runs; 0: split plan (S = p.splits, groups)
  int groups;
  int* err;
};

// stream-K: CTA c of G owns units [c U / G, (c + 1) U / G)
__host__ __device__ __forceinline__ int sk_begin(int c, long long U, int G) {
  return (int)((long long)c * U / G);
}
__host__ __device__ __forceinline__ int sk_owner(int u, long long U, int G) {
  int o = (int)((long long)u * G / U);
  while (o + 1 < G && sk_begin(o + 1, U, G) <= u) ++o;
  while (o > 0 && sk_begin(o, U, G) > u) --o;
  return o;
}

// segment i of CTA c: tile, k-block range [kb_lo, kb_hi], the CTA's slot among
// the tile's contributors and their number
struct Seg {
  int tile, kb_lo, kb_hi, slot, n;
};

struct Sched {
  int stream_k, nkb, tiles, G, S, groups;
  long long U;
  int u0, u1;  // stream-K run of this CTA
  __host__ __device__ Sched(int sk, int N, int K, int G_, int S_, int groups_, int c)
      : stream_k(sk), nkb(K / 128), tiles(N / 128), G(G_), S(S_), groups(groups_) {
    U = (long long)tiles * nkb;
    u0 = sk_begin(c, U, G);
    u1 = sk_begin(c + 1, U, G);
  }
  __host__ __device__ int count(int c) const {
    if (stream_k) return u1 > u0 ? (u1 - 1) / nkb - u0 / nkb + 1 : 0;
    const int g = c / S;
    return tiles > g ? (tiles - g + groups - 1) / groups : 0;
  }
  __host__ __device__ Seg get(int c, int i) const {
    Seg sg;
    if (stream_k) {
      const int t0 = u0 / nkb, t1 = (u1 - 1) / nkb;
      sg.tile = t0 + i;
      sg.kb_lo = i == 0 ? u0 % nkb : 0;
      sg.kb_hi = sg.tile == t1 ? (u1 - 1) % nkb : nkb - 1;
      const int first = sk_owner(sg.tile * nkb, U, G);
      sg.slot = c - first;
      sg.n = sk_owner(sg.tile * nkb + nkb - 1, U, G) - first + 1;
    } else {
      const int split = c % S;
      sg.tile = c / S + i * groups;
      sg.kb_lo = split * nkb / S;
      sg.kb_hi = (split + 1) * nkb / S - 1;
      sg.slot = split;
      sg.n = S;
    }
    return sg;
  }
};

// Fused epilogue for one activation row m of tile `tile` (a warp; lane owns
// EPC consecutive channels).  v / u hold the integer sums of the row's limbs
// (exact up to the fp32 conversion); the row's power-of-two scale and the
// channel scales turn them into the W8A16 product.
template <int MODE>
__device__ __forceinline__ void w8_epilogue_row(const W8Params& p, int tile, int m, int lane,
                                                float (&v)[4], float (&u)[4]) {
  constexpr int EPC = (MODE == kSiluMul) ? 2 : 4;
  const int gch = tile * 128 + lane * EPC;
  const float rs = __ldg(p.xscale + m);
#pragma unroll
  for (int e = 0; e < EPC; ++e) v[e] *= __ldg(p.scale + gch + e) * rs;
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
    if (p.hmax_out) {
      const float4 nw = __ldg(reinterpret_cast<const float4*>(p.next_norm + gch));
      float mw = fmaxf(fmaxf(fabsf(hv.x * nw.x), fabsf(hv.y * nw.y)), fmaxf(fabsf(hv.z * nw.z), fabsf(hv.w * nw.w)));
      mw = warp_max(mw);
      if (lane == 0) p.hmax_out[(size_t)tile * p.M + m] = mw;
    }
  } else if (MODE == kSiluMul) {
    float o[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float gv = v[e];
      const float uv = u[e] * (__ldg(p.scale + gch + 64 + e) * rs);
      o[e] = (gv / (1.0f + expf(-gv))) * uv;
    }
    *reinterpret_cast<float2*>(p.act + (size_t)m * (p.N / 2) + tile * 64 + lane * 2) = make_float2(o[0], o[1]);
    if (p.amax_out) {
      const float mx = warp_max(fmaxf(fabsf(o[0]), fabsf(o[1])));
      if (lane == 0) p.amax_out[(size_t)tile * p.M + m] = mx;
    }
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
      const KvSeq sq = p.kv.seq[bi];
      const int lrow = sq.n0 + (p.kv.seq[bi + 1].ctx_start - sq.ctx_start) + j;
      const int slot = kv_slot(p.kv, lrow, sq.rs_pre);
      dstp = base + (((size_t)sq.cseq * p.n_kv_heads + kvh) * p.kv.slots + slot) * 128;
    }
    *reinterpret_cast<uint2*>(dstp + lane * 4) = o;
  }
}

template <int MP, int MODE>
__global__ void __launch_bounds__(WI_THREADS, 1)
    w8i_kernel(const __grid_constant__ CUtensorMap map_x, const WiArgs args) {
  using C = WiCfg<MP>;
  const W8Params& p = args.p;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;                                         // [NS][W block | limb tile]
  float* red = reinterpret_cast<float*>(smem + C::NS * C::STAGE);  // [MP][129]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::NS * C::STAGE + C::RED_BYTES);
  uint64_t* empty = full + C::NS;
  uint64_t* accf = empty + C::NS;  // [2]
  uint64_t* acce = accf + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int nkb = p.K / 128;
  const int c = blockIdx.x;
  const Sched sch(args.stream_k, p.N, p.K, gridDim.x, p.splits, args.groups, c);
  const int nseg = sch.count(c);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
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
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // The weights depend on nothing earlier in the stream: the first NS ring
      // stages get their weight blocks before this kernel waits for the
      // previous one (programmatic dependent launch); their limb tiles follow
      // once it has completed.
      int pre_kb[C::NS];
      int it = 0;
      bool ok = true, waited = false;
      auto release_prefetch = [&](int n) {
        griddep_wait();
        waited = true;
        for (int j = 0; j < n; ++j)
          tma_load_2d(ring + j * C::STAGE + WI_WB, &map_x, &full[j], pre_kb[j] * 128, 0);
      };
      for (int i = 0; i < nseg && ok; ++i) {
        const Seg sg = sch.get(c, i);
        for (int kb = sg.kb_lo; kb <= sg.kb_hi; ++kb, ++it) {
          const int s = it % C::NS;
          if (it == C::NS) release_prefetch(C::NS);
          if (!mbar_wait(&empty[s], ((it / C::NS) & 1) ^ 1, args.err, abort_flag)) { ok = false; break; }
          uint8_t* st = ring + s * C::STAGE;
          mbar_arrive_expect_tx(&full[s], C::STAGE);
          bulk_load(st, args.w_tiles + ((size_t)sg.tile * nkb + kb) * WI_WB, WI_WB, &full[s]);
          if (it < C::NS)
            pre_kb[it] = kb;
          else
            tma_load_2d(st + WI_WB, &map_x, &full[s], kb * 128, 0);
        }
      }
      if (!waited) release_prefetch(it < C::NS ? it : C::NS);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_s8(128, C::NB);
      int it = 0;
      bool ok = true;
      for (int i = 0; i < nseg && ok; ++i) {
        const Seg sg = sch.get(c, i);
        const int b = i & 1;  // take a free accumulator
        if (!mbar_wait(&acce[b], ((i >> 1) & 1) ^ 1, args.err, abort_flag)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * C::ACC_COLS;
        for (int kb = sg.kb_lo; kb <= sg.kb_hi; ++kb, ++it) {
          const int s = it % C::NS;
          if (!mbar_wait(&full[s], (it / C::NS) & 1, args.err, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = umma_desc_sw128(smem_u32(ring + s * C::STAGE));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(ring + s * C::STAGE + WI_WB));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_i8(acc, adesc + 2 * k, bdesc + 2 * k, idesc, (kb == sg.kb_lo && k == 0) ? 0u : 1u);
          umma_commit(&empty[s]);
        }
        umma_commit(&accf[b]);
      }
    }
  } else {
    // epilogue warps -> TMEM lane quadrant warp % 4 (= channels q*32 ..)
    griddep_wait();  // the epilogue reads and writes what earlier kernels touch
    const int q = warp & 3;
    const int et = threadIdx.x - 64;  // 0..127
    constexpr int EPC = (MODE == kSiluMul) ? 2 : 4;
    // No epilogue warp leaves the loop early: after a timeout (the abort flag)
    // the segments are walked without work, so every named barrier below is
    // reached by all four warps and every tile counter returns to zero.
    for (int seg = 0; seg < nseg; ++seg) {
      const int b = seg & 1;
      const Seg sg = sch.get(c, seg);
      const int tile = sg.tile;
      const bool whole = sg.n == 1;
      const bool live = mbar_wait(&accf[b], (seg >> 1) & 1, args.err, abort_flag) && !*abort_flag;
      if (live) tc_fence_after();
      // accumulator column l * MP + m holds limb l of row m: recombine
      float r[MP];
#pragma unroll
      for (int m = 0; m < MP; ++m) r[m] = 0.f;
      const uint32_t tb = tmem + b * C::ACC_COLS + ((uint32_t)(q * 32) << 16);
#pragma unroll
      for (int c0 = 0; c0 < MP && live; c0 += 32) {
        uint32_t a0[32], a1[32], a2[32];
        tmem_ld32(tb + c0, a0);
        tmem_ld32(tb + MP + c0, a1);
        tmem_ld32(tb + 2 * MP + c0, a2);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (c0 + e < MP)
            r[c0 + e] = fmaf((float)(int)a2[e], 16384.f, fmaf((float)(int)a1[e], 128.f, (float)(int)a0[e]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[b]);  // accumulator free for segment seg + 2
      const int ch = q * 32 + lane;
      if (whole) {
        // own tile: stage the accumulator in shared memory rows and run the epilogue
#pragma unroll
        for (int m = 0; m < MP; ++m) red[m * 129 + ch] = r[m];
        named_bar(1, 128);
        for (int m = q; m < p.M && live; m += 4) {
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
        // partial -> the tile's slot, coalesced per row
        const int n_seg = sg.n;
        float* dst = args.part + ((size_t)tile * args.maxseg + sg.slot) * MP * 128;
#pragma unroll
        for (int m = 0; m < MP; ++m) dst[m * 128 + ch] = r[m];
        __threadfence();
        named_bar(1, 128);
        // The contributors that finish together merge the tile together: each
        // waits (bounded) for every partial, then sums the slots of its share
        // of the rows in slot order (deterministic) and runs the fused
        // epilogue on them.  In the split plan every contributor takes part
        // (equal K slices).  In stream-K the tile is the last segment of every
        // contributor's run but possibly the highest one's, whose run goes on
        // into the next tile: that one only leaves its partial, so no SM is
        // held back from the next kernel.  The counter counts the n_seg
        // arrivals, then the participants' departures; the last departure
        // resets it.  With one CTA taking all 32 rows the merge tail was
        // ~10 us.
        int npart = n_seg, pidx = sg.slot;
        if (args.stream_k) {
          const int last_owner = sk_owner(tile * nkb + nkb - 1, sch.U, sch.G);
          const bool last_late = (sk_begin(last_owner + 1, sch.U, sch.G) - 1) / nkb == tile;
          npart = n_seg - (last_late ? 0 : 1);
          pidx = seg == nseg - 1 ? sg.slot : -1;
        }
        const int r0 = pidx >= 0 ? pidx * p.M / npart : 0;
        const int r1 = pidx >= 0 ? (pidx + 1) * p.M / npart : 0;
        if (et == 0) {
          atomicAdd(args.counters + tile, 1);
          bool arrived = pidx >= 0;
          for (uint32_t i = 0; arrived && ld_acquire_gpu(args.counters + tile) < n_seg; ++i) {
            if (i >= kSpinLimit || *abort_flag) {
              if (!*abort_flag) atomicExch(args.err, kDevMbarTimeout);
              *abort_flag = 1;
              arrived = false;
              break;
            }
            __nanosleep(32);
          }
          *last_flag = arrived;
        }
        named_bar(1, 128);
        if (*last_flag) {
          __threadfence();
          const float* src = args.part + (size_t)tile * args.maxseg * MP * 128;
          // two rows per pass, every slot's partial loaded before any add
          for (int m0 = r0 + q; m0 < r1 && live; m0 += 8) {
            float4 va[2][8], ua[2][8];
#pragma unroll
            for (int rr = 0; rr < 2; ++rr)
#pragma unroll
              for (int s = 0; s < 8; ++s) {
                const int m = m0 + 4 * rr;
                va[rr][s] = make_float4(0.f, 0.f, 0.f, 0.f);
                ua[rr][s] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (s < n_seg && m < r1) {
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
              if (m < r1) {
                float v[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int s = 0; s < 8; ++s) {  // fixed slot order: deterministic
                  v[0] += va[rr][s].x; v[1] += va[rr][s].y; v[2] += va[rr][s].z; v[3] += va[rr][s].w;
                  u[0] += ua[rr][s].x; u[1] += ua[rr][s].y;
                }
                w8_epilogue_row<MODE>(p, tile, m, lane, v, u);
              }
            }
          }
        }
        named_bar(1, 128);
        if (pidx >= 0 && et == 0 && atomicAdd(args.counters + tile, 1) == n_seg + npart - 1)
          args.counters[tile] = 0;  // every participant is done with the tile
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

// ------------------------------------------------------------------ weight packing
// Source row r (int8 [n_src, K] row-major) becomes output channel
// d = (r / grp) * gstride + r % grp + base (concatenation / gate|up interleave)
// and is stored tile-major, [d / 128][k / 128][d % 128][128 B], with the
// 16-byte chunk j of row d % 128 at position j ^ (d % 8): every (tile, k128)
// block is one contiguous 16 KB run already in the UMMA 128-byte swizzle.
__global__ void w8_tilepack_kernel(const int8_t* __restrict__ src, int n_src, int K,
                                   int8_t* __restrict__ dst, int grp, int gstride, int base) {
  const int cpr = K / 16;
  const int nkb = K / 128;
  const size_t total = (size_t)n_src * cpr;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int r = idx / cpr, c = idx % cpr;
    const int d = (r / grp) * gstride + r % grp + base;
    const int kb = c / 8, j = c % 8, row = d % 128;
    const size_t off = (((size_t)(d / 128) * nkb + kb) * 128 + row) * 128 + ((j ^ (row & 7)) << 4);
    *reinterpret_cast<uint4*>(dst + off) = reinterpret_cast<const uint4*>(src + (size_t)r * K)[c];
  }
}

// ------------------------------------------------------------------ activation limbs
// Limb layout of one launch: int8 [3][MP][K] (limb-major), rows M..MP-1 zero,
// plus the fp32 row scale 2^(e_m - 20) with max|x_m| < 2^e_m (limbs_of).

__device__ __forceinline__ float block_max(float v, float* sh) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    t = warp_max(t);
    if (threadIdx.x == 0) sh[32] = t;
  }
  __syncthreads();
  return sh[32];
}

// f16 or fp32 rows -> limbs.  With producer maxima (maxpart [nparts, M]) every CTA
// converts one 1024-element chunk of one row in a single pass; without them a
// CTA owns a whole row and finds its maximum first.
constexpr int LB_CHUNK = 1024;

__device__ __forceinline__ void limbs_store4(int8_t* o0, int8_t* o1, int8_t* o2, int k,
                                             const float (&v)[4], float up) {
  int8_t l[3][4];
#pragma unroll
  for (int t = 0; t < 4; ++t) limbs_of(v[t], up, l[0][t], l[1][t], l[2][t]);
  *reinterpret_cast<char4*>(o0 + k) = make_char4(l[0][0], l[0][1], l[0][2], l[0][3]);
  *reinterpret_cast<char4*>(o1 + k) = make_char4(l[1][0], l[1][1], l[1][2], l[1][3]);
  *reinterpret_cast<char4*>(o2 + k) = make_char4(l[2][0], l[2][1], l[2][2], l[2][3]);
}

__device__ __forceinline__ void load_h4(const __half* row, int k, float (&v)[4]) {
  const uint2 raw = *reinterpret_cast<const uint2*>(row + k);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void load_h4(const float* row, int k, float (&v)[4]) {
  const float4 a = *reinterpret_cast<const float4*>(row + k);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}

// max over the producer's partials of row m (every thread of the CTA gets it)
__device__ __forceinline__ float part_max(const float* part, int nparts, int M, int m, float* sh) {
  float mx = 0.f;
  for (int q = threadIdx.x; q < nparts; q += blockDim.x) mx = fmaxf(mx, part[(size_t)q * M + m]);
  return block_max(mx, sh);
}

template <class T>
__global__ void w8_limbs_kernel(const T* __restrict__ x, int M, int MP, int K,
                                const float* __restrict__ maxpart, int nparts,
                                int8_t* __restrict__ xl, float* __restrict__ xscale) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float sh[33];
  const int m = blockIdx.y;
  const int k0 = maxpart ? blockIdx.x * LB_CHUNK : 0;
  const int k1 = maxpart ? min(K, k0 + LB_CHUNK) : K;
  int8_t* o0 = xl + (size_t)m * K;
  int8_t* o1 = o0 + (size_t)MP * K;
  int8_t* o2 = o1 + (size_t)MP * K;
  if (m >= M) {
    for (int k = k0 + threadIdx.x * 4; k < k1; k += blockDim.x * 4) {
      *reinterpret_cast<uint32_t*>(o0 + k) = 0u;
      *reinterpret_cast<uint32_t*>(o1 + k) = 0u;
      *reinterpret_cast<uint32_t*>(o2 + k) = 0u;
    }
    if (threadIdx.x == 0 && blockIdx.x == 0) xscale[m] = 1.f;
    return;
  }
  const T* row = x + (size_t)m * K;
  // with producer maxima, this thread's first four elements are loaded before
  // the maximum's reduction waits
  const int kf = k0 + threadIdx.x * 4;
  float v0[4] = {0.f, 0.f, 0.f, 0.f};
  if (maxpart && kf < k1) load_h4(row, kf, v0);
  float mx;
  if (maxpart) {
    mx = part_max(maxpart, nparts, M, m, sh);
  } else {
    mx = 0.f;
    for (int k = threadIdx.x * 4; k < K; k += blockDim.x * 4) {
      float v[4];
      load_h4(row, k, v);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3]))));
    }
    mx = block_max(mx, sh);
  }
  int e;
  frexpf(mx, &e);  // every |x| <= mx < 2^e
  const float up = ldexpf(1.f, 20 - e);
  if (threadIdx.x == 0 && blockIdx.x == 0) xscale[m] = ldexpf(1.f, e - 20);
  for (int k = kf; k < k1; k += blockDim.x * 4) {
    float v[4] = {v0[0], v0[1], v0[2], v0[3]};
    if (!maxpart || k != kf) load_h4(row, k, v);
    limbs_store4(o0, o1, o2, k, v, up);
  }
}

// RMSNorm of the residual rows (h fp32; sums of h^2 and maxima of |h * w| from
// the producer's partials) split into limbs straight from fp32 -- no f16
// rounding, so no f16 range limit and 21 significant bits near the row
// maximum; one 1024-element chunk of one row per CTA
__global__ void rmsnorm_limbs_kernel(const float* __restrict__ h, const float* __restrict__ hstat,
                                     const float* __restrict__ hmax, int hparts, int M, int MP, int K,
                                     const float* __restrict__ w, float eps, int8_t* __restrict__ xl,
                                     float* __restrict__ xscale) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float sh[33], shm[33];
  const int m = blockIdx.y;
  const int k0 = blockIdx.x * LB_CHUNK, k1 = min(K, k0 + LB_CHUNK);
  int8_t* o0 = xl + (size_t)m * K;
  int8_t* o1 = o0 + (size_t)MP * K;
  int8_t* o2 = o1 + (size_t)MP * K;
  if (m >= M) {
    for (int k = k0 + threadIdx.x * 4; k < k1; k += blockDim.x * 4) {
      *reinterpret_cast<uint32_t*>(o0 + k) = 0u;
      *reinterpret_cast<uint32_t*>(o1 + k) = 0u;
      *reinterpret_cast<uint32_t*>(o2 + k) = 0u;
    }
    if (threadIdx.x == 0 && blockIdx.x == 0) xscale[m] = 1.f;
    return;
  }
  // Every load of the CTA is issued before any reduction waits: the producer's
  // partial sums and maxima of row m, and this thread's first four elements of
  // the row and of the norm weight (one pass covers the chunk when
  // LB_CHUNK = 4 * blockDim.x).
  const float* row = h + (size_t)m * K;
  const int kf = k0 + threadIdx.x * 4;
  float4 hv0 = make_float4(0.f, 0.f, 0.f, 0.f), wv0 = hv0;
  if (kf < k1) {
    hv0 = *reinterpret_cast<const float4*>(row + kf);
    wv0 = __ldg(reinterpret_cast<const float4*>(w + kf));
  }
  float ss = 0.f, mx = 0.f;
  for (int q = threadIdx.x; q < hparts; q += blockDim.x) {
    ss += hstat[(size_t)q * M + m];
    mx = fmaxf(mx, hmax[(size_t)q * M + m]);
  }
  ss = warp_sum(ss);
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) {
    sh[threadIdx.x >> 5] = ss;
    shm[threadIdx.x >> 5] = mx;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const bool in = threadIdx.x < (blockDim.x >> 5);
    float t = in ? sh[threadIdx.x] : 0.f;
    float u = in ? shm[threadIdx.x] : 0.f;
    t = warp_sum(t);
    u = warp_max(u);
    if (threadIdx.x == 0) {
      sh[32] = rsqrtf(t / static_cast<float>(K) + eps);
      shm[32] = u;
    }
  }
  __syncthreads();
  const float rstd = sh[32];
  // bound on max |h * rstd * w|: the fp32 products stay within 2^-9 of
  // rstd * max |h * w|
  const float bound = shm[32] * rstd * (1.f + 1.f / 512.f);
  int e;
  frexpf(bound, &e);
  const float up = ldexpf(1.f, 20 - e);
  if (threadIdx.x == 0 && blockIdx.x == 0) xscale[m] = ldexpf(1.f, e - 20);
  for (int k = kf; k < k1; k += blockDim.x * 4) {
    const float4 hv = k == kf ? hv0 : *reinterpret_cast<const float4*>(row + k);
    const float4 wv = k == kf ? wv0 : __ldg(reinterpret_cast<const float4*>(w + k));
    const float v[4] = {hv.x * rstd * wv.x, hv.y * rstd * wv.y, hv.z * rstd * wv.z, hv.w * rstd * wv.w};
    limbs_store4(o0, o1, o2, k, v, up);
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

// limb tensor int8 [rows][K], box [rows][128 B] with the 128-byte swizzle
static bool map_i8_rows(CUtensorMap* m, const void* base, uint64_t K, uint64_t rows) {
  EncodeTiledFn2 enc = encode_fn();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15) || K % 128 || rows > 256) return false;
  cuuint64_t dims[2] = {K, rows};
  cuuint64_t strides[1] = {K};
  cuuint32_t box[2] = {128, (cuuint32_t)rows};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Split plan: S in 1..8 and groups = floor(SMs / S) from a small cost model
// (a slice streams nkb/S blocks of 16 KB at ~42 GB/s per SM; S > 1 adds a
// merge of ~4 us per tile, hidden behind the next tile's stream when that is
// longer, exposed once at the end). Returns the estimate in us.
static constexpr double kW8BlockUs = 16384.0 / 42e3;
static double w8i_split_plan(int tiles, int nkb, int num_sms, int* splits, int* groups) {
  const double t_kb = kW8BlockUs;
  double best = 1e30;
  int bs = 1, bg = num_sms < tiles ? num_sms : tiles;
  for (int s = 1; s <= 8 && s <= nkb; ++s) {
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
  return best;
}

// The launch schedule: grid size, split plan, stream-K or not, partial slots.
struct W8Schedule {
  int grid, splits, groups, stream_k, maxseg;
};

static W8Schedule w8i_schedule(int N, int K, int num_sms) {
  const int tiles = N / 128, nkb = K / 128;
  W8Schedule w{};
  int splits = 1, groups = 1;
  const double split_est = w8i_split_plan(tiles, nkb, num_sms, &splits, &groups);
  // Stream-K for long K, and for wide shapes (at least one tile per SM) whose
  // split plan ends on a poorly filled round: there the even share of the
  // units, ceil(U / SMs) block times plus the shared merge, is shorter.
  // Narrow shapes keep the split plan; their many 3-4-way shared tiles merge
  // slower than this estimate says.
  const long long units = (long long)tiles * nkb;
  const double sk_est = (double)((units + num_sms - 1) / num_sms) * kW8BlockUs + 4.0;
  if (nkb >= 64 || (tiles >= num_sms && sk_est < split_est - 1e-9)) {
    // stream-K: one CTA per SM (never more CTAs than units), shrunk until no
    // tile is shared by more than 8 CTAs
    const long long U = units;
    int G = (int)std::min<long long>(num_sms, U);
    for (;;) {
      int ms = 1;
      for (int t = 0; t < tiles; ++t)
        ms = std::max(ms, sk_owner(t * nkb + nkb - 1, U, G) - sk_owner(t * nkb, U, G) + 1);
      if (ms <= 8 || G == 1) {
        w.grid = G; w.splits = G; w.groups = 1; w.stream_k = 1; w.maxseg = ms;
        return w;
      }
      --G;
    }
  }
  w.splits = splits;
  w.groups = groups;
  w.grid = w.splits * w.groups;
  w.stream_k = 0;
  w.maxseg = w.splits;
  return w;
}

size_t w8tc_part_floats(int N, int K, int M, int num_sms) {
  const W8Schedule w = w8i_schedule(N, K, num_sms);
  const int mp = (M + 15) / 16 * 16;
  return (size_t)(N / 128) * w.maxseg * mp * 128;
}

template <int MP, int MODE>
static cudaError_t w8i_launch_t(const CUtensorMap& mx, const WiArgs& a, cudaStream_t st) {
  using C = WiCfg<MP>;
  const size_t smem = C::SMEM;
  auto kern = w8i_kernel<MP, MODE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  DFL_TRY(max_smem_carveout(kern));
  return launch_pdl(kern, dim3(a.stream_k ? a.p.splits : a.p.splits * a.groups), dim3(WI_THREADS), smem,
                    st, mx, a);
}

template <int MODE>
static cudaError_t w8i_mode(const CUtensorMap& mx, const WiArgs& a, int mp, cudaStream_t st) {
  if (mp == 16) return w8i_launch_t<16, MODE>(mx, a, st);
  if (mp == 32) return w8i_launch_t<32, MODE>(mx, a, st);
  if (mp == 48) return w8i_launch_t<48, MODE>(mx, a, st);
  return w8i_launch_t<64, MODE>(mx, a, st);
}

cudaError_t w8tc_launch(const int8_t* w_tiles, const W8Params& pin, int mode, int* err, float* part,
                        size_t part_floats, int* counters, int num_sms, cudaStream_t st) {
  if (pin.M < 1 || pin.M > 64 || pin.N % 128 || pin.K % 128 || !pin.xl || !pin.xscale)
    return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(w_tiles) & 15) return cudaErrorInvalidValue;
  W8Params p = pin;
  const W8Schedule w = w8i_schedule(p.N, p.K, num_sms);
  p.splits = w.splits;  // stream-K: the grid size; split plan: S
  const int mp = (p.M + 15) / 16 * 16;
  if (!part || !counters || part_floats < (size_t)(p.N / 128) * w.maxseg * mp * 128)
    return cudaErrorInvalidValue;
  CUtensorMap mx;
  if (!map_i8_rows(&mx, p.xl, p.K, 3 * mp)) return cudaErrorInvalidValue;
  WiArgs a{p, w_tiles, part, counters, w.maxseg, w.stream_k, w.groups, err};
  if (mode == kQKV) return w8i_mode<kQKV>(mx, a, mp, st);
  if (mode == kResid) return w8i_mode<kResid>(mx, a, mp, st);
  if (mode == kSiluMul) return w8i_mode<kSiluMul>(mx, a, mp, st);
  if (mode == kStore) return w8i_mode<kStore>(mx, a, mp, st);
  return cudaErrorInvalidValue;
}

cudaError_t w8_tilepack_launch(const int8_t* src, int n_src, int K, int8_t* dst, int grp, int gstride,
                               int base, cudaStream_t st) {
  if (K % 128) return cudaErrorInvalidValue;
  w8_tilepack_kernel<<<1024, 256, 0, st>>>(src, n_src, K, dst, grp, gstride, base);
  return cudaGetLastError();
}

template <class T>
static cudaError_t w8_limbs_go(const T* x, int M, int K, const float* maxpart, int nparts, int8_t* xl,
                               float* xscale, cudaStream_t st) {
  if (M < 1 || M > 64 || K % 128) return cudaErrorInvalidValue;
  const int mp = (M + 15) / 16 * 16;
  const dim3 grid(maxpart ? (K + LB_CHUNK - 1) / LB_CHUNK : 1, mp);
  DFL_TRY(max_smem_carveout(w8_limbs_kernel<T>));
  return launch_pdl(w8_limbs_kernel<T>, grid, dim3(256), 0, st, x, M, mp, K, maxpart, nparts, xl, xscale);
}
cudaError_t w8_limbs_launch(const __half* x, int M, int K, const float* maxpart, int nparts,
                            int8_t* xl, float* xscale, cudaStream_t st) {
  return w8_limbs_go(x, M, K, maxpart, nparts, xl, xscale, st);
}
cudaError_t w8_limbs_launch(const float* x, int M, int K, const float* maxpart, int nparts,
                            int8_t* xl, float* xscale, cudaStream_t st) {
  return w8_limbs_go(x, M, K, maxpart, nparts, xl, xscale, st);
}

cudaError_t rmsnorm_limbs_launch(const float* h, const float* hstat, const float* hmax, int hparts,
                                 int M, int K, const float* w, float eps, int8_t* xl, float* xscale,
                                 cudaStream_t st) {
  if (M < 1 || M > 64 || K % 128 || !hmax) return cudaErrorInvalidValue;
  const int mp = (M + 15) / 16 * 16;
  const dim3 grid((K + LB_CHUNK - 1) / LB_CHUNK, mp);
  DFL_TRY(max_smem_carveout(rmsnorm_limbs_kernel));
  return launch_pdl(rmsnorm_limbs_kernel, grid, dim3(256), 0, st, h, hstat, hmax, hparts, M, mp, K, w, eps,
                    xl, xscale);
}

}  // namespace dfl
