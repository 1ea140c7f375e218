// Non-causal GQA block attention on the 5th-gen tensor cores (dflash.py:310-319).
//
// Same split-KV decomposition and partial format as attention.cu: one CTA per
// (KV split, kv head, sequence) holds all R = G * block query rows of the kv
// head (G = NQ / NKV), so each K/V row is read from HBM once, and writes an
// unnormalised partial (O, m, l) that attn_combine_kernel merges in a fixed
// order.  Here both products run on tcgen05 with the accumulators in TMEM:
//
//   S_g = Q_g K_j^T     M=128 query rows, N=64 kv rows, K=128 (kind::f16)
//   O_g += P_g V_j      M=128, N=128 head dims, K=64 kv rows (V as an
//                       MN-major operand: kv rows of 128-byte d chunks)
//
// The query rows are padded to NG groups of 128 (NG = 1 or 2).
// Roles:
//   warps 0 .. 4NG-1  softmax, one thread per query row (TMEM lane).  Each
//       thread reads its S row, computes base-2 exponents and the running sum,
//       and writes P (f16) into shared memory in the UMMA 128-byte swizzle.
//       O is rescaled in TMEM only when the running max grows by more than 2^8
//       (P then stays below 256, exact enough in f16), so most tiles need no
//       O traffic.
//   4 producer warps  cp.async of the K/V tiles, each row through the KvMap
//       (cache rings), into the swizzled stages of a 3-stage ring; a tile is
//       signalled once the next one is issued (two tiles in flight).
//   1 MMA warp        single-thread issue.  Order per tile: S_0, S_1, then
//       PV_0 and the next S_0 once P_0 is ready, PV_1 ... so the softmax of one
//       group overlaps the MMAs of the other.
// Every mbarrier wait is bounded; a timeout sets the error word and unwinds.
#include "kernels.cuh"

namespace dfl {

constexpr int TA_TK = 64;                  // kv rows per tile
constexpr int TA_NS = 3;                   // K/V stages
constexpr int TA_PROD = 4;                 // producer warps
constexpr int TA_KV_BYTES = TA_TK * 256;   // K (or V) of one tile: 64 rows x 128 f16
constexpr int TA_STAGE = 2 * TA_KV_BYTES;  // K then V
constexpr int TA_QG = 128 * 256;           // one query group: 128 rows x 128 f16
constexpr int TA_PG = 128 * 128;           // P of one group: 128 rows x 64 f16
constexpr float TA_RESCALE = 8.0f;         // log2 of the largest P before O is rescaled

template <int NG>
struct TaCfg {
  static constexpr int SOFT_WARPS = 4 * NG;
  static constexpr int PROD_WARP0 = SOFT_WARPS;
  static constexpr int MMA_WARP = SOFT_WARPS + TA_PROD;
  static constexpr int THREADS = 32 * (MMA_WARP + 1);
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = NG * TA_QG;
  static constexpr int P_OFF = KV_OFF + TA_NS * TA_STAGE;
  static constexpr int BAR_OFF = P_OFF + NG * TA_PG;
  static constexpr size_t SMEM = (size_t)BAR_OFF + 256 + 1024;
  static constexpr uint32_t S_COL = 0;        // S_g at g * 64
  static constexpr uint32_t O_COL = NG * 64;  // O_g at O_COL + g * 128
  static constexpr uint32_t TMEM_COLS = NG == 1 ? 256 : 512;
};

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
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

template <int NG>
__global__ void __launch_bounds__(TaCfg<NG>::THREADS, 1) attn_tc_kernel(const AttnParams p) {
  using C = TaCfg<NG>;
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + TA_NS;
  uint64_t* s_ready = empty + TA_NS;  // [NG]
  uint64_t* p_ready = s_ready + NG;   // [NG]
  uint64_t* o_ready = p_ready + NG;   // [NG]
  uint64_t* q_ready = o_ready + NG;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_ready + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int split = blockIdx.x, kvh = blockIdx.y, bi = blockIdx.z;
  const int G = p.nq / p.nkv;
  const int R = G * p.block;
  const bool mapped = p.kv.nseq > 0;
  const int kv_len = mapped ? p.kv.n_att[bi] : p.kv_len;
  const int rs = mapped ? p.kv.rs_post[bi] : 0;
  const int kv0 = split * p.chunk;
  const int kv1 = min(kv_len, kv0 + p.chunk);
  const int ntiles = kv1 > kv0 ? (kv1 - kv0 + TA_TK - 1) / TA_TK : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t pbase = (((size_t)bi * p.nkv + kvh) * p.splits + split) * (size_t)R;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TA_NS; ++s) {
      mbar_init(&full[s], 32 * TA_PROD);
      mbar_init(&empty[s], 1);
    }
    for (int g = 0; g < NG; ++g) {
      mbar_init(&s_ready[g], 1);
      mbar_init(&p_ready[g], 128);
      mbar_init(&o_ready[g], 1);
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

  if (warp >= C::PROD_WARP0 && warp < C::MMA_WARP) {
    // ---- producers: Q once, then the K/V tiles (rows through the KvMap)
    const int t = threadIdx.x - 32 * C::PROD_WARP0;  // 0..127
    const __half* qg = p.q + ((size_t)bi * p.nq + (size_t)kvh * G) * p.block * 128;
    for (int idx = t; idx < NG * 128 * 16; idx += 32 * TA_PROD) {
      const int r = idx >> 4, c = idx & 15;  // 16-byte piece c of the 256-byte row r
      const int g = r >> 7, rr = r & 127, ch = c >> 3, cc = c & 7;
      uint8_t* dst = smem + C::Q_OFF + g * TA_QG + ch * (128 * 128) + rr * 128 + ((cc ^ (rr & 7)) << 4);
      cp_async16_zfill(smem_u32(dst), qg + (size_t)min(r, R - 1) * 128 + c * 8, r < R);
    }
    cp_async_commit();
    cp_async_wait<0>();
    fence_proxy_async_smem();
    mbar_arrive(q_ready);
    const __half* kg = p.k + ((size_t)bi * p.nkv + kvh) * (size_t)p.kv_cap * 128;
    const __half* vg = p.v + ((size_t)bi * p.nkv + kvh) * (size_t)p.kv_cap * 128;
    int issued = 0;
    for (int j = 0; j < ntiles; ++j) {
      const int s = j % TA_NS;
      if (!mbar_wait(&empty[s], ((j / TA_NS) & 1) ^ 1, p.err, abort_flag)) break;
      uint8_t* st = smem + C::KV_OFF + s * TA_STAGE;
      for (int idx = t; idx < TA_TK * 16; idx += 32 * TA_PROD) {
        const int r = idx >> 4, c = idx & 15, ch = c >> 3, cc = c & 7;
        const int row = kv0 + j * TA_TK + r;
        const bool ok = row < kv1;
        const int lrow = ok ? row : kv0;  // a valid address even when nothing is read
        const size_t off = (size_t)(mapped ? kv_slot(p.kv, lrow, rs) : lrow) * 128 + c * 8;
        const int sw = ch * (TA_TK * 128) + r * 128 + ((cc ^ (r & 7)) << 4);
        cp_async16_zfill(smem_u32(st + sw), kg + off, ok);
        cp_async16_zfill(smem_u32(st + TA_KV_BYTES + sw), vg + off, ok);
      }
      cp_async_commit();
      ++issued;
      // tile j-1 has landed once at most one copy group (tile j) is in flight.
      // Signalling one tile behind keeps two tiles in flight and never holds a
      // tile back that the MMA needs before it can free a stage.
      if (j >= 1) {
        cp_async_wait<1>();
        fence_proxy_async_smem();
        mbar_arrive(&full[(j - 1) % TA_NS]);
      }
    }
    cp_async_wait<0>();
    fence_proxy_async_smem();
    if (issued > 0) mbar_arrive(&full[(issued - 1) % TA_NS]);
  } else if (warp == C::MMA_WARP) {
    // ---- single-thread MMA issue
    if (lane == 0 && ntiles > 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(128, TA_TK, 0);
      constexpr uint32_t idesc_o = umma_idesc_f16(128, 128, 0) | (1u << 16);  // B (V) MN-major
      const uint32_t qa = smem_u32(smem + C::Q_OFF), kva = smem_u32(smem + C::KV_OFF),
                     pa = smem_u32(smem + C::P_OFF);
      auto issue_s = [&](int g, int s) {
        for (int kk = 0; kk < 8; ++kk) {
          const int ch = kk >> 2, w = kk & 3;
          const uint64_t ad = umma_desc_sw128(qa + g * TA_QG + ch * (128 * 128)) + 2 * w;
          const uint64_t bd = umma_desc_sw128(kva + s * TA_STAGE + ch * (TA_TK * 128)) + 2 * w;
          umma_f16(tmem + C::S_COL + g * TA_TK, ad, bd, idesc_s, kk > 0);
        }
      };
      auto issue_pv = [&](int g, int s, bool acc) {
        for (int ks = 0; ks < TA_TK / 16; ++ks) {
          const uint64_t ad = umma_desc_sw128(pa + g * TA_PG) + 2 * ks;
          const uint64_t bd = umma_desc_sw128_mn(kva + s * TA_STAGE + TA_KV_BYTES + ks * 2048, TA_TK * 128);
          umma_f16(tmem + C::O_COL + g * 128, ad, bd, idesc_o, (acc || ks > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_ready, 0, p.err, abort_flag) && mbar_wait(&full[0], 0, p.err, abort_flag);
      if (ok) {
        tc_fence_after();
        for (int g = 0; g < NG; ++g) {
          issue_s(g, 0);
          umma_commit(&s_ready[g]);
        }
      }
      for (int j = 0; j < ntiles && ok; ++j) {
        const int s = j % TA_NS, s1 = (j + 1) % TA_NS;
        for (int g = 0; g < NG && ok; ++g) {
          if (!mbar_wait(&p_ready[g], j & 1, p.err, abort_flag)) { ok = false; break; }
          tc_fence_after();
          issue_pv(g, s, j > 0);
          if (g == NG - 1) umma_commit(&empty[s]);  // every read of stage s is issued
          if (j + 1 < ntiles) {
            if (g == 0) {
              if (!mbar_wait(&full[s1], ((j + 1) / TA_NS) & 1, p.err, abort_flag)) { ok = false; break; }
              tc_fence_after();
            }
            issue_s(g, s1);
            umma_commit(&s_ready[g]);
          } else {
            umma_commit(&o_ready[g]);
          }
        }
      }
    }
  } else {
    // ---- softmax: thread = query row g * 128 + r (TMEM lane r of group g)
    const int g = warp >> 2;
    const int r = 32 * (warp & 3) + lane;
    const int qrow = g * 128 + r;
    const bool valid = qrow < R;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const uint32_t s_t = tmem + C::S_COL + g * TA_TK + lane_off;
    const uint32_t o_t = tmem + C::O_COL + g * 128 + lane_off;
    uint8_t* prow = smem + C::P_OFF + g * TA_PG + r * 128;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      if (!mbar_wait(&s_ready[g], j & 1, p.err, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t a[32], b[32];
      tmem_ld32(s_t, a);
      tmem_ld32(s_t + 32, b);
      tmem_ld_wait();
      const int nvalid = kv1 - (kv0 + j * TA_TK);  // >= 1
      float sv[TA_TK];
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < TA_TK; ++e) {
        float v = __uint_as_float(e < 32 ? a[e] : b[e - 32]) * p.scale_log2;
        if (e >= nvalid) v = -INFINITY;
        sv[e] = v;
        mx = fmaxf(mx, v);
      }
      // rescale O only when the max has grown by more than 2^8 (warp-uniform
      // TMEM traffic; lanes that need no rescale multiply by 1)
      const bool grow = mx > m_used + TA_RESCALE;
      const float m_new = grow ? mx : m_used;
      if (__any_sync(0xffffffffu, grow) && j > 0) {
        // O holds tiles < j: PV(j-1) was issued before S(j), so it is complete
        const float f = grow ? exp2f(m_used - m_new) : 1.f;
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
      uint32_t pk[TA_TK / 2];
#pragma unroll
      for (int e = 0; e < TA_TK; e += 2) {
        const float p0 = exp2f(sv[e] - m_used), p1 = exp2f(sv[e + 1] - m_used);
        l += p0 + p1;
        pk[e / 2] = pack_f16x2(p0, p1);
      }
#pragma unroll
      for (int cc = 0; cc < 8; ++cc)
        *reinterpret_cast<uint4*>(prow + ((cc ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * cc], pk[4 * cc + 1], pk[4 * cc + 2], pk[4 * cc + 3]);
      fence_proxy_async_smem();  // P visible to the tensor core
      tc_fence_before();
      mbar_arrive(&p_ready[g]);
    }
    float* orow = p.opart + (pbase + (valid ? qrow : 0)) * 128;
    if (ntiles == 0 || !ok) {
      if (valid) {
        for (int d = 0; d < 128; d += 4) *reinterpret_cast<float4*>(orow + d) = make_float4(0.f, 0.f, 0.f, 0.f);
        p.mpart[pbase + qrow] = -INFINITY;
        p.lpart[pbase + qrow] = 0.f;
      }
    } else if (mbar_wait(&o_ready[g], 0, p.err, abort_flag)) {
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
  tc_fence_before();
  __syncthreads();
  if (warp == C::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int NG>
static cudaError_t attn_tc_launch_t(const AttnParams& p, int batch, cudaStream_t st) {
  using C = TaCfg<NG>;
  auto kern = attn_tc_kernel<NG>;
  DFL_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
  DFL_TRY(max_smem_carveout(kern));
  return launch_pdl(kern, dim3(p.splits, p.nkv, batch), dim3(C::THREADS), C::SMEM, st, p);
}

cudaError_t attn_tc_launch(const AttnParams& p, int batch, __half* out, cudaStream_t st) {
  const int G = p.nq / p.nkv;
  const int R = G * p.block;
  if (p.nq % p.nkv || R < 1 || R > 256 || p.kv_len < 1 || p.chunk % TA_TK || p.normrope)
    return cudaErrorInvalidValue;
  DFL_TRY(R <= 128 ? attn_tc_launch_t<1>(p, batch, st) : attn_tc_launch_t<2>(p, batch, st));
  return attn_combine_launch(p, batch, out, st);
}

}  // namespace dfl
