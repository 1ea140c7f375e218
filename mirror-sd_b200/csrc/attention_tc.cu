// Non-causal GQA block attention on the 5th-gen tensor cores (dflash.py:310-319).
//
// Same split-KV decomposition and partial format as attention.cu: one CTA per
// (KV split, kv head, sequence) holds all R = G * block query rows of the kv
// head (G = NQ / NKV), so each K/V row is read from HBM once, and writes an
// unnormalised partial (O, m, l) that attn_combine_kernel merges in a fixed
// order.  Here both products run on tcgen05 with the accumulators in TMEM:
//
//   S_g = Q_g K_j^T     M=128 query rows, N=64 kv rows, K=128 (kind::f16)
//   O_g += P_g V_j      M=128, N=128 head dims, K=64 kv rows; P is the A
//                       operand straight from TMEM (f16 pairs written over
//                       its own S columns), V the B operand from shared
//                       memory as an MN-major tile (kv rows of 128-byte d
//                       chunks)
//
// The query rows are padded to NG groups of 128 (NG = 1 or 2).  S/P is
// double-buffered in TMEM per group, so the MMAs of tile j+1 run while the
// softmax works on tile j, and with P out of shared memory the K/V ring gets
// every byte that Q leaves (5 or 6 stages in flight).
// Roles:
//   warps 0 .. 4NG-1  softmax, one thread per query row (TMEM lane).  Each
//       thread reads its S row, computes base-2 exponents (an FMA per element,
//       one f16x2 ex2 per pair) and the running sum, and stores P into its
//       TMEM lane.  O is rescaled in TMEM only when
//       the running max grows by more than 2^8 (P then stays below 256), so
//       most tiles need no O traffic.  Warps whose 32 rows are all padding
//       take no part.  Group 1's real rows sit in its top lanes, so its
//       softmax warps share no scheduler with group 0's first warp.
//   3 producer warps  K/V tiles into the swizzled stages of the ring.  A full
//       tile whose 64 rows sit in 64 consecutive slots (always in the
//       stateless forward; in a cache ring except at the sink / wrap
//       boundaries) is one TMA copy per 64-column half, completed by
//       transaction bytes, so NS tiles stay in flight.  Other tiles are
//       copied row by row through the KvMap with cp.async, zero-filling the
//       rows past the end (stale V rows must not reach P.V).
//   2 MMA warps       one issuing thread each, on different schedulers:
//       S(j) of every group (warp 4NG + 4, scheduler 0) and PV(j) of every
//       group once its P is ready (warp 4NG + 1, scheduler 1).  A single
//       issuing thread spent about a third of each tile on its own waits,
//       commits and fences with the tensor pipe idle.
// Every mbarrier wait is bounded; a timeout sets the error word and unwinds.
#include "kernels.cuh"

namespace dfl {

constexpr int TA_TK = 64;                  // kv rows per tile
constexpr int TA_PROD = 3;                 // producer warps
constexpr int TA_KV_BYTES = TA_TK * 256;   // K (or V) of one tile: 64 rows x 128 f16
constexpr int TA_STAGE = 2 * TA_KV_BYTES;  // K then V
constexpr int TA_QG = 128 * 256;           // one query group: 128 rows x 128 f16
constexpr float TA_RESCALE = 8.0f;         // log2 of the largest P before O is rescaled

// NS_ 0: the deepest K/V ring shared memory allows (one CTA per SM); 2: a
// double buffer small enough for two CTAs per SM, for grids with many CTAs
// per SM (many sequences), where the second CTA hides the per-tile latency.
// HALVES 2 (one group of at most 64 query rows): the group's rows are loaded
// twice, as MMA rows 0-63 and 64-127, and the softmax warps of the upper copy
// take kv columns 32-63 of every tile while the lower copy takes columns
// 0-31, each with its own running max and sum (P is zero in the other
// half's columns); the two halves are merged once at the end.  All four
// softmax warps work instead of two, on half the columns each.
template <int NG, int NS_ = 0, int HALVES = 1>
struct TaCfg {
  static constexpr int NS = NS_ ? NS_ : (NG == 1 ? 6 : 5);  // K/V stages
  // registers per thread: two CTAs of THREADS threads must fit in 64K
  static constexpr int MAX_REGS = NS_ == 2 ? 112 : 255;
  static constexpr int SOFT_WARPS = 4 * NG;
  // Warp w issues on scheduler w % 4.  The two MMA-issuing warps sit on
  // different schedulers: the PV warp (which also owns the TMEM allocation)
  // on scheduler 1, the S warp on scheduler 0.  The producers are warps
  // PROD_WARP0 (the TMA issuer), PROD_WARP0 + 2 and PROD_WARP0 + 3.
  static constexpr int PROD_WARP0 = SOFT_WARPS;
  static constexpr int MMA_WARP = SOFT_WARPS + 1;
  static constexpr int S_WARP = SOFT_WARPS + 4;
  static constexpr int THREADS = 32 * (SOFT_WARPS + TA_PROD + 2);
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = NG * TA_QG;
  static constexpr int BAR_OFF = KV_OFF + NS * TA_STAGE;
  static constexpr size_t SMEM = (size_t)BAR_OFF + 256 + 1024;
  static constexpr uint32_t S_COL = 0;            // S/P[g][buffer] at (2g + buffer) * 64
  static constexpr uint32_t O_COL = NG * 2 * 64;  // O_g at O_COL + g * 128
  static constexpr uint32_t TMEM_COLS = NG == 1 ? 256 : 512;
};

// D (TMEM) += A (TMEM, K-major, f16 pairs per column) . B (shared-memory descriptor)
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// SW128 descriptor of an MN-major operand: 64-element (128-byte) MN chunks
// lbo_bytes apart, 8-row K groups 1024 bytes apart
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFF) >> 4);
  d |= (uint64_t)(lbo_bytes >> 4) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// map_k / map_v: [batch * NKV planes][kv_cap slots][128] f16, box 64 x 64 x 1
// (the producer's named barrier is the non-aligned form: lane 0 can still be
// waiting on a stage while its warp-mates arrive)

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// max of three (exact, like two fmaxf)
__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// (a0, a1) * (b, b) + (c, c) as one packed fp32 FMA: two fmaf, rounded alike
__device__ __forceinline__ float2 ffma2_bc(float a0, float a1, float b, float c) {
  uint64_t x, y, z, r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(y) : "f"(b));
  asm("mov.b64 %0, {%1, %1};" : "=l"(z) : "f"(c));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(x), "l"(y), "l"(z));
  float2 o;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(o.x), "=f"(o.y) : "l"(r));
  return o;
}
// two base-2 exponentials in one MUFU op: the f16 pair ex2(x0), ex2(x1)
__device__ __forceinline__ uint32_t ex2_f16x2(float x0, float x1) {
  const uint32_t a = pack_f16x2(x0, x1);
  uint32_t y;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(a));
  return y;
}
__device__ __forceinline__ uint32_t hadd2_u(uint32_t a, uint32_t b) {
  uint32_t y;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(y) : "r"(a), "r"(b));
  return y;
}

template <int NG, int NS_, int HALVES>
__global__ void __launch_bounds__(TaCfg<NG, NS_, HALVES>::THREADS) __maxnreg__((TaCfg<NG, NS_, HALVES>::MAX_REGS))
    attn_tc_kernel(const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v,
                   const AttnParams p) {
  using C = TaCfg<NG, NS_, HALVES>;
  constexpr int TA_NS = C::NS;
  static_assert(HALVES == 1 || NG == 1, "column halves need a single query group");
  // The producer warps wait for the previous kernel only after requesting the
  // K/V tiles that kernel cannot have written (below); every other warp waits
  // here, before it touches global memory.
  const bool prod_warp = (threadIdx.x >> 5) >= C::PROD_WARP0 && (threadIdx.x >> 5) != C::MMA_WARP &&
                         (threadIdx.x >> 5) != C::S_WARP;
  if (!prod_warp) griddep_wait();
  griddep_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + TA_NS;
  uint64_t* s_ready = empty + TA_NS;    // [2] S(j) of every group in TMEM buffer j & 1 (one commit)
  // P(j) stored over S(j) by every group, per buffer j & 1: one barrier for
  // all groups, so the PV thread waits once per tile.  PV(j) complete is
  // empty[j % TA_NS] (the stage's last reader), which the softmax also waits
  // on before it rescales O.
  uint64_t* p_ready = s_ready + 2;      // [2]
  uint64_t* o_ready = p_ready + 2;       // [NG]
  uint64_t* q_ready = o_ready + NG;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_ready + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int split = blockIdx.x, kvh = blockIdx.y, bi = blockIdx.z;
  const int G = p.nq / p.nkv;
  const int R = G * p.block;
  const bool mapped = p.kv.nseq > 0;
  const int kv_len = mapped ? p.kv.seq[bi].n_att : p.kv_len;
  const int rs = mapped ? p.kv.seq[bi].rs_post : 0;
  const int kv0 = split * p.chunk;
  const int kv1 = min(kv_len, kv0 + p.chunk);
  const int ntiles = kv1 > kv0 ? (kv1 - kv0 + TA_TK - 1) / TA_TK : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Group 1's real rows occupy its top TMEM lanes (g1_shift = 128 - those rows
  // rounded up to 32), so with 32 of them their softmax warp is warp 7, on
  // scheduler 3, not on scheduler 0 beside group 0's first softmax warp.
  const int g1_shift = NG == 2 ? 128 - (R - 128 + 31) / 32 * 32 : 0;
  const size_t pbase = (((size_t)bi * p.nkv + kvh) * p.splits + split) * (size_t)R;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TA_NS; ++s) {
      mbar_init(&full[s], 1);  // producer thread 0 (with the TMA bytes, or after cp.async)
      mbar_init(&empty[s], 1);
    }
    int nthr = 0;
    for (int g = 0; g < NG; ++g) {
      // softmax threads of group g: its warps holding at least one real row
      // (with halves: rows 0-63 twice)
      const int rows = min(128, R - g * 128);
      nthr += HALVES == 2 ? 64 * ((rows + 31) / 32) : 32 * ((rows + 31) / 32);
      mbar_init(&o_ready[g], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_ready[b], 1);
      mbar_init(&p_ready[b], nthr);
    }
    mbar_init(q_ready, 32 * TA_PROD);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == C::MMA_WARP) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (prod_warp) {
    // ---- producers: Q once, then the K/V tiles (rows through the KvMap)
    const int pw = warp == C::PROD_WARP0 ? 0 : warp - C::PROD_WARP0 - 1;
    const int t = 32 * pw + lane;  // 0..127
    const int kseq = mapped ? p.kv.seq[bi].cseq : bi;   // K/V store sequence
    const int plane = kseq * p.nkv + kvh;
    // The previous kernel writes Q and this forward's block rows of K/V, the
    // last p.block logical rows; the context rows come from the context K|V
    // GEMM, which completed before that kernel could start.  So whole,
    // contiguous tiles below the block rows go to the ring (one per stage, at
    // most TA_NS) before the dependency wait, while the previous kernel drains.
    int npre = 0;
    {
      const int pre_end = kv_len - p.block;
      for (int j = 0; j < ntiles && j < TA_NS; ++j) {
        const int row0 = kv0 + j * TA_TK;
        if (row0 + TA_TK > kv1 || row0 + TA_TK > pre_end) break;
        const int slot0 = mapped ? kv_slot(p.kv, row0, rs) : row0;
        if ((mapped ? kv_slot(p.kv, row0 + TA_TK - 1, rs) : row0 + TA_TK - 1) != slot0 + TA_TK - 1) break;
        if (t == 0) {
          uint8_t* st = smem + C::KV_OFF + j * TA_STAGE;
          mbar_arrive_expect_tx(&full[j], TA_STAGE);
          for (int ch = 0; ch < 2; ++ch) {
            tma_load_3d(st + ch * (TA_TK * 128), &map_k, &full[j], ch * 64, slot0, plane);
            tma_load_3d(st + TA_KV_BYTES + ch * (TA_TK * 128), &map_v, &full[j], ch * 64, slot0, plane);
          }
        }
        ++npre;
      }
    }
    griddep_wait();
    const __half* qg = p.q + ((size_t)bi * p.nq + (size_t)kvh * G) * p.block * 128;
    for (int idx = t; idx < NG * 128 * 16; idx += 32 * TA_PROD) {
      const int r = idx >> 4, c = idx & 15;  // 16-byte piece c of the 256-byte row r
      const int g = r >> 7, rr = r & 127, ch = c >> 3, cc = c & 7;
      uint8_t* dst = smem + C::Q_OFF + g * TA_QG + ch * (128 * 128) + rr * 128 + ((cc ^ (rr & 7)) << 4);
      // halves: MMA rows 64-127 repeat rows 0-63; group 1 sits g1_shift lanes up
      const int src = HALVES == 2 ? (r & 63) : g == 1 ? r - g1_shift : r;
      const bool real = src < R && (g == 0 || rr >= g1_shift);
      cp_async16_zfill(smem_u32(dst), qg + (size_t)max(0, min(src, R - 1)) * 128 + c * 8, real);
    }
    cp_async_commit();
    cp_async_wait<0>();
    fence_proxy_async_smem();
    mbar_arrive(q_ready);

    const __half* kg = p.k + ((size_t)kseq * p.nkv + kvh) * (size_t)p.kv_cap * 128;
    const __half* vg = p.v + ((size_t)kseq * p.nkv + kvh) * (size_t)p.kv_cap * 128;
    // Producer thread 0 alone waits for free stages and issues the TMA tiles;
    // the other producer threads sleep on a named barrier and join only for the
    // tiles copied row by row.  Nobody leaves the loop early: every producer
    // thread reaches the same named barriers, and after a timeout (thread 0's
    // `dead`) the copies are skipped while the bounded waits elsewhere unwind.
    bool dead = false;
    for (int j = npre; j < ntiles; ++j) {
      const int s = j % TA_NS;
      uint8_t* st = smem + C::KV_OFF + s * TA_STAGE;
      const int row0 = kv0 + j * TA_TK;
      const int slot0 = mapped ? kv_slot(p.kv, row0, rs) : row0;
      const bool whole = row0 + TA_TK <= kv1;
      // consecutive slots: the map is piecewise consecutive and every break
      // (sink -> ring, ring wrap) changes the end-to-end distance
      const bool contig = whole && (mapped ? kv_slot(p.kv, row0 + TA_TK - 1, rs) : row0 + TA_TK - 1) ==
                                       slot0 + TA_TK - 1;
      if (t == 0 && !dead && !mbar_wait(&empty[s], ((j / TA_NS) & 1) ^ 1, p.err, abort_flag)) dead = true;
      if (contig) {
        if (t == 0 && !dead) {
          mbar_arrive_expect_tx(&full[s], TA_STAGE);
          for (int ch = 0; ch < 2; ++ch) {
            tma_load_3d(st + ch * (TA_TK * 128), &map_k, &full[s], ch * 64, slot0, plane);
            tma_load_3d(st + TA_KV_BYTES + ch * (TA_TK * 128), &map_v, &full[s], ch * 64, slot0, plane);
          }
        }
      } else {
        named_bar_sync(1, 32 * TA_PROD);  // thread 0 has seen the stage free
        if (!*abort_flag) {
          for (int idx = t; idx < TA_TK * 16; idx += 32 * TA_PROD) {
            const int r = idx >> 4, c = idx & 15, ch = c >> 3, cc = c & 7;
            const int row = row0 + r;
            const bool ok = row < kv1;
            const int lrow = ok ? row : kv0;  // a valid address even when nothing is read
            const size_t off = (size_t)(mapped ? kv_slot(p.kv, lrow, rs) : lrow) * 128 + c * 8;
            const int sw = ch * (TA_TK * 128) + r * 128 + ((cc ^ (r & 7)) << 4);
            cp_async16_zfill(smem_u32(st + sw), kg + off, ok);
            cp_async16_zfill(smem_u32(st + TA_KV_BYTES + sw), vg + off, ok);
          }
          cp_async_commit();
          cp_async_wait<0>();  // rare (partial or boundary tiles): no overlap needed
          fence_proxy_async_smem();
        }
        named_bar_sync(1, 32 * TA_PROD);
        if (t == 0 && !dead) mbar_arrive(&full[s]);
      }
    }
  } else if (warp == C::MMA_WARP || warp == C::S_WARP) {
    // ---- MMA issue by two single threads on different schedulers, so the
    // waits, commits and fences of one overlap the other's queued MMAs:
    //   S warp:  S(j) of every group once stage j is full and PV(j-2), the
    //            last reader of S/P buffer j & 1, has completed;
    //   PV warp: PV(j) of every group once P(j) is stored, then the stage's
    //            free barrier, which also tells the softmax that O holds PV(j).
    // MMAs of one thread execute in issue order; across the two threads the
    // only hazards are the S/P buffer (above), stage reuse (S(j) completes
    // before P(j) exists, hence before PV(j) frees the stage) and O, which
    // only the PV thread writes.
    if (lane == 0 && ntiles > 0) {
      const uint32_t qa = smem_u32(smem + C::Q_OFF), kva = smem_u32(smem + C::KV_OFF);
      bool ok = mbar_wait(q_ready, 0, p.err, abort_flag);
      if (warp == C::S_WARP) {
        constexpr uint32_t idesc_s = umma_idesc_f16(128, TA_TK, 0);
        // k-step kk (16 head dims) of S_g = Q_g K^T
        auto issue_s_step = [&](int g, int s, int b, int kk) {
          const int ch = kk >> 2, w = kk & 3;
          const uint64_t ad = umma_desc_sw128(qa + g * TA_QG + ch * (128 * 128)) + 2 * w;
          const uint64_t bd = umma_desc_sw128(kva + s * TA_STAGE + ch * (TA_TK * 128)) + 2 * w;
          umma_f16(tmem + C::S_COL + (2 * g + b) * TA_TK, ad, bd, idesc_s, kk > 0);
        };
        for (int j = 0; j < ntiles && ok; ++j) {
          const int s = j % TA_NS, b = j & 1;
          if (!mbar_wait_ready(&full[s], (j / TA_NS) & 1, p.err, abort_flag)) break;
          // (empty[(j - 2) % TA_NS] next completes with PV(j - 2 + TA_NS),
          // which needs S(j - 2 + TA_NS) from this thread: no parity alias)
          if (j >= 2 && !mbar_wait_ready(&empty[(j - 2) % TA_NS], ((j - 2) / TA_NS) & 1, p.err, abort_flag))
            break;
          tc_fence_after();
          // the two groups' k-steps alternate, so consecutive MMAs accumulate
          // into different TMEM buffers
          for (int kk = 0; kk < 8; ++kk)
            for (int g = 0; g < NG; ++g) issue_s_step(g, s, b, kk);
          umma_commit(&s_ready[b]);
        }
      } else {
        constexpr uint32_t idesc_o = umma_idesc_f16(128, 128, 0) | (1u << 16);  // B (V) MN-major
        // k-step ks (16 kv rows) of O_g += P_g V: P as 8 TMEM columns of f16 pairs
        auto issue_pv_step = [&](int g, int s, int b, bool acc, int ks) {
          const uint32_t pt = tmem + C::S_COL + (2 * g + b) * TA_TK + ks * 8;
          const uint64_t bd = umma_desc_sw128_mn(kva + s * TA_STAGE + TA_KV_BYTES + ks * 2048, TA_TK * 128);
          umma_f16_ts(tmem + C::O_COL + g * 128, pt, bd, idesc_o, (acc || ks > 0) ? 1u : 0u);
        };
        for (int j = 0; j < ntiles && ok; ++j) {
          const int s = j % TA_NS, b = j & 1;
          if (!mbar_wait_ready(&p_ready[b], (j >> 1) & 1, p.err, abort_flag)) break;
          tc_fence_after();
          for (int ks = 0; ks < TA_TK / 16; ++ks)
            for (int g = 0; g < NG; ++g) issue_pv_step(g, s, b, j > 0, ks);
          if (j == ntiles - 1)
            for (int g = 0; g < NG; ++g) umma_commit(&o_ready[g]);
          umma_commit(&empty[s]);  // every read of stage s, and PV(j), is issued
        }
      }
    }
  } else {
    // ---- softmax: thread = TMEM lane r of group g.  Without halves it owns
    // query row g * 128 + r; with halves, lanes r and r + 64 own row r & 63,
    // lanes below 64 taking kv columns 0-31 of every tile and the others 32-63
    const int g = warp >> 2;
    const int r = 32 * (warp & 3) + lane;
    constexpr int CW = TA_TK / HALVES;  // kv columns per thread and tile
    const int half = HALVES == 2 ? (r >> 6) : 0;
    const int coff = half * CW;
    const int qrow = HALVES == 2 ? (r & 63) : g * 128 + r - (g == 1 ? g1_shift : 0);
    const bool valid = qrow < R && (g == 0 || r >= g1_shift);
    // the warp holds a real row
    const bool active = HALVES == 2 ? ((32 * (warp & 3)) & 63) < R
                                    : (g == 0 || 32 * (warp & 3) >= g1_shift) &&
                                          g * 128 + 32 * (warp & 3) - (g == 1 ? g1_shift : 0) < R;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const uint32_t o_t = tmem + C::O_COL + g * 128 + lane_off;
    const float c = p.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles && active; ++j) {
      const int b = j & 1;
      if (!mbar_wait(&s_ready[b], (j >> 1) & 1, p.err, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t sv[CW];
      const uint32_t s_t = tmem + C::S_COL + (2 * g + b) * TA_TK + lane_off;
      if (HALVES == 2) {
        uint32_t a[32];
        tmem_ld32(s_t + coff, a);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < CW; ++e) sv[e] = a[e];
      } else {
        uint32_t a[32], bb[32];
        tmem_ld32(s_t, a);
        tmem_ld32(s_t + 32, bb);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          sv[e] = a[e];
          sv[(32 + e) % CW] = bb[e];
        }
      }
      // valid columns in this thread's range (can be <= 0 for the upper half of a short tile)
      const int nvalid = kv1 - (kv0 + j * TA_TK) - coff;
      float mx = -INFINITY;
      const bool full_tile = nvalid >= CW;
      if (full_tile) {
        // four interleaved chains (the max is exact in any order)
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int e = 0; e < CW; e += 2)
          m4[(e >> 1) & 3] = fmax3f(m4[(e >> 1) & 3], __uint_as_float(sv[e]), __uint_as_float(sv[e + 1]));
        mx = fmax3f(fmaxf(m4[0], m4[1]), m4[2], m4[3]);
      } else {
#pragma unroll
        for (int e = 0; e < CW; ++e)
          if (e < nvalid) mx = fmaxf(mx, __uint_as_float(sv[e]));
      }
      // scores in base-2 units: s * c with c = log2(e) / sqrt(128) > 0, so the
      // max commutes with the scaling
      const float m_cand = mx * c;
      const bool grow = m_cand > m_used + TA_RESCALE;
      const float m_new = grow ? m_cand : m_used;
      if (__any_sync(0xffffffffu, grow) && j > 0) {
        // O must hold tiles < j before it is rescaled
        // (empty[(j - 1) % TA_NS] completes with PV(j - 1); its next phase
        // needs P(j - 1 + TA_NS), so the parity cannot alias)
        if (!mbar_wait(&empty[(j - 1) % TA_NS], ((j - 1) / TA_NS) & 1, p.err, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const float f = grow ? ex2_approx(m_used - m_new) : 1.f;
#pragma unroll 1
        for (int cblk = 0; cblk < 4; ++cblk) {
          uint32_t o[32];
          tmem_ld32(o_t + cblk * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
          tmem_st32(o_t + cblk * 32, o);
        }
        tmem_st_wait();
        l *= f;
      }
      m_used = m_new;
      // P = 2^(s c - m) two at a time in f16 (the MMA consumes f16 P anyway);
      // masked columns get -inf, hence 0, and with halves the other half's
      // columns are 0.  The row sum adds f16 pairs in groups of 8 (at most
      // 8 * 256, exact to 2^-10) and then in fp32.
      uint32_t own[CW / 2];
      const float neg_m = -m_used;
      if (full_tile) {
#pragma unroll
        for (int e = 0; e < CW; e += 2) {
          const float2 x = ffma2_bc(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1]), c, neg_m);
          own[e / 2] = ex2_f16x2(x.x, x.y);
        }
      } else {
#pragma unroll
        for (int e = 0; e < CW; e += 2) {
          const float x0 = e < nvalid ? fmaf(__uint_as_float(sv[e]), c, neg_m) : -INFINITY;
          const float x1 = e + 1 < nvalid ? fmaf(__uint_as_float(sv[e + 1]), c, neg_m) : -INFINITY;
          own[e / 2] = ex2_f16x2(x0, x1);
        }
      }
      uint32_t pk[TA_TK / 2];
#pragma unroll
      for (int i = 0; i < TA_TK / 2; ++i) pk[i] = (i / (CW / 2) == half) ? own[i % (CW / 2)] : 0u;
#pragma unroll
      for (int q = 0; q < TA_TK / 2; q += 4) {
        const uint32_t s4 = hadd2_u(hadd2_u(pk[q], pk[q + 1]), hadd2_u(pk[q + 2], pk[q + 3]));
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&s4));
        l += f.x + f.y;
      }
      // P over the first 32 columns of this S buffer (its S values are read)
      tmem_st32(s_t, pk);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_ready[b]);
    }
    if (HALVES == 2) {
      // merge the halves: the upper copy hands (O, m, l) to the lower one
      // through shared memory (the K/V stages: every MMA that read them has
      // completed once O is final), laid out [column][row] for the banks
      float* xo = reinterpret_cast<float*>(smem + C::KV_OFF);
      float* xm = xo + 128 * 64;
      float* xl = xm + 64;
      const bool have = __all_sync(0xffffffffu, active && ntiles > 0 && ok &&
                                                    mbar_wait(&o_ready[g], 0, p.err, abort_flag));
      if (have) tc_fence_after();
      if (half == 1 && active) {
#pragma unroll 1
        for (int cblk = 0; cblk < 4; ++cblk) {
          uint32_t o[32];
          if (have) {
            tmem_ld32(o_t + cblk * 32, o);
            tmem_ld_wait();
          }
#pragma unroll
          for (int e = 0; e < 32; ++e) xo[(cblk * 32 + e) * 64 + qrow] = have ? __uint_as_float(o[e]) : 0.f;
        }
        xm[qrow] = have ? m_used : -INFINITY;
        xl[qrow] = have ? l : 0.f;
      }
      named_bar_sync(3, 128);
      if (half == 0 && active) {
        const float ma = have ? m_used : -INFINITY, mb = xm[qrow];
        const float mm = fmaxf(ma, mb);
        const float wa = ma == -INFINITY ? 0.f : exp2f(ma - mm);
        const float wb = mb == -INFINITY ? 0.f : exp2f(mb - mm);
        const float lsum = (have ? l : 0.f) * wa + xl[qrow] * wb;
        const int hq = qrow / p.block, jr = qrow - hq * p.block;
        const int head = kvh * G + hq;
        __half* dst = p.out ? p.out + ((size_t)bi * p.block + jr) * ((size_t)p.nq * 128) + (size_t)head * 128
                            : nullptr;
        float* orow = p.opart + (pbase + (valid ? qrow : 0)) * 128;
        const float inv = lsum > 0.f ? 1.0f / lsum : 0.f;
        float amax = 0.f;
#pragma unroll 1
        for (int cblk = 0; cblk < 4; ++cblk) {
          uint32_t o[32];
          if (have) {
            tmem_ld32(o_t + cblk * 32, o);
            tmem_ld_wait();
          }
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e)
            v[e] = (have ? __uint_as_float(o[e]) * wa : 0.f) + xo[(cblk * 32 + e) * 64 + qrow] * wb;
          if (!valid) continue;
          if (dst) {
            uint32_t h2[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              h2[e / 2] = pack_f16x2(v[e] * inv, v[e + 1] * inv);
              const float2 back = __half22float2(*reinterpret_cast<const __half2*>(&h2[e / 2]));
              amax = fmaxf(amax, fmaxf(fabsf(back.x), fabsf(back.y)));
            }
            uint4* d4 = reinterpret_cast<uint4*>(dst + cblk * 32);
#pragma unroll
            for (int w4 = 0; w4 < 4; ++w4)
              d4[w4] = make_uint4(h2[4 * w4], h2[4 * w4 + 1], h2[4 * w4 + 2], h2[4 * w4 + 3]);
          } else {
#pragma unroll
            for (int e = 0; e < 32; e += 4)
              *reinterpret_cast<float4*>(orow + cblk * 32 + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
          }
        }
        if (valid) {
          if (dst) {
            if (p.omax) p.omax[(size_t)head * gridDim.z * p.block + (size_t)bi * p.block + jr] = amax;
          } else {
            p.mpart[pbase + qrow] = mm;
            p.lpart[pbase + qrow] = lsum;
          }
        }
      }
    } else {
    float* orow = p.opart + (pbase + (valid ? qrow : 0)) * 128;
    if (!active) {
      // padding rows only: nothing to write
    } else if (ntiles == 0 || !ok) {
      if (valid && p.out) {
        const int hq = qrow / p.block, jr = qrow - hq * p.block;
        __half* dst = p.out + ((size_t)bi * p.block + jr) * ((size_t)p.nq * 128) + (size_t)(kvh * G + hq) * 128;
        for (int d = 0; d < 128; d += 8) *reinterpret_cast<uint4*>(dst + d) = make_uint4(0, 0, 0, 0);
        if (p.omax) p.omax[(size_t)(kvh * G + hq) * gridDim.z * p.block + (size_t)bi * p.block + jr] = 0.f;
      } else if (valid) {
        for (int d = 0; d < 128; d += 4) *reinterpret_cast<float4*>(orow + d) = make_float4(0.f, 0.f, 0.f, 0.f);
        p.mpart[pbase + qrow] = -INFINITY;
        p.lpart[pbase + qrow] = 0.f;
      }
    } else if (p.out && mbar_wait(&o_ready[g], 0, p.err, abort_flag)) {
      // one split: O / l is the attention row, stored as f16 where the
      // combine would put it (row bi * block + j, columns head * 128 ..),
      // with the head's max |out| for the o-projection's limb split
      tc_fence_after();
      const int hq = qrow / p.block, jr = qrow - hq * p.block;
      const int head = kvh * G + hq;
      __half* dst = p.out + ((size_t)bi * p.block + jr) * ((size_t)p.nq * 128) + (size_t)head * 128;
      const float inv = 1.0f / l;
      float amax = 0.f;
#pragma unroll 1
      for (int cblk = 0; cblk < 4; ++cblk) {
        uint32_t o[32];
        tmem_ld32(o_t + cblk * 32, o);
        tmem_ld_wait();
        if (valid) {
          uint32_t h2[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            h2[e / 2] = pack_f16x2(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv);
            const float2 back = __half22float2(*reinterpret_cast<const __half2*>(&h2[e / 2]));
            amax = fmaxf(amax, fmaxf(fabsf(back.x), fabsf(back.y)));
          }
          uint4* d4 = reinterpret_cast<uint4*>(dst + cblk * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) d4[v] = make_uint4(h2[4 * v], h2[4 * v + 1], h2[4 * v + 2], h2[4 * v + 3]);
        }
      }
      if (valid && p.omax) p.omax[(size_t)head * gridDim.z * p.block + (size_t)bi * p.block + jr] = amax;
    } else if (!p.out && mbar_wait(&o_ready[g], 0, p.err, abort_flag)) {
      tc_fence_after();
#pragma unroll 1
      for (int cblk = 0; cblk < 4; ++cblk) {
        uint32_t o[32];
        tmem_ld32(o_t + cblk * 32, o);
        tmem_ld_wait();
        if (valid) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(orow + cblk * 32 + e) =
                make_float4(__uint_as_float(o[e]), __uint_as_float(o[e + 1]), __uint_as_float(o[e + 2]),
                            __uint_as_float(o[e + 3]));
        }
      }
      if (valid) {
        p.mpart[pbase + qrow] = m_used;
        p.lpart[pbase + qrow] = l;
      }
    }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == C::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

typedef CUresult (*EncodeTiledFnA)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [planes][slots][128] f16 -> box 64 x 64 x 1 with the 128-byte swizzle
static bool map_kv(CUtensorMap* m, const void* base, uint64_t slots, uint64_t planes) {
  static EncodeTiledFnA enc = nullptr;
  if (!enc) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return false;
    enc = reinterpret_cast<EncodeTiledFnA>(ptr);
  }
  if (reinterpret_cast<uintptr_t>(base) & 15) return false;
  cuuint64_t dims[3] = {128, slots, planes};
  cuuint64_t strides[2] = {256, slots * 256};
  cuuint32_t box[3] = {64, (cuuint32_t)TA_TK, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NG, int NS_, int HALVES>
static cudaError_t attn_tc_launch_t(const AttnParams& p, int batch, cudaStream_t st) {
  using C = TaCfg<NG, NS_, HALVES>;
  auto kern = attn_tc_kernel<NG, NS_, HALVES>;
  CUtensorMap mk, mv;
  const uint64_t planes = (uint64_t)(p.kv.nseq > 0 ? p.kv_seqs : batch) * p.nkv;
  if (planes < (uint64_t)batch * p.nkv || !map_kv(&mk, p.k, p.kv_cap, planes) || !map_kv(&mv, p.v, p.kv_cap, planes))
    return cudaErrorInvalidValue;
  DFL_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
  DFL_TRY(max_smem_carveout(kern));
  return launch_pdl(kern, dim3(p.splits, p.nkv, batch), dim3(C::THREADS), C::SMEM, st, mk, mv, p);
}

cudaError_t attn_tc_launch(const AttnParams& p, int batch, __half* out, cudaStream_t st, AttnLimbOut* limbs) {
  const int G = p.nq / p.nkv;
  const int R = G * p.block;
  if (p.nq % p.nkv || R < 1 || R > 256 || p.kv_len < 1 || p.chunk % TA_TK || p.normrope)
    return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  DFL_TRY(cudaGetDevice(&dev));
  DFL_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const long long ctas = (long long)p.splits * p.nkv * batch;
  AttnParams q = p;
  q.out = p.splits == 1 ? out : nullptr;   // one split: the kernel writes the rows itself
  const bool many = ctas >= 2LL * sms;   // two CTAs per SM pay off
  cudaError_t e;
  if (R > 128)
    e = attn_tc_launch_t<2, 0, 1>(q, batch, st);
  else if (R <= 64)
    e = many ? attn_tc_launch_t<1, 2, 2>(q, batch, st) : attn_tc_launch_t<1, 0, 2>(q, batch, st);
  else
    e = many ? attn_tc_launch_t<1, 2, 1>(q, batch, st) : attn_tc_launch_t<1, 0, 1>(q, batch, st);
  DFL_TRY(e);
  if (q.out) return cudaSuccess;
  if (limbs && p.nq <= 64) {  // the merge writes the o-projection's limbs
    DFL_TRY(attn_combine_limbs_launch(p, batch, *limbs, st));
    limbs->done = true;
    return cudaSuccess;
  }
  return attn_combine_launch(p, batch, out, st);
}

}  // namespace dfl
