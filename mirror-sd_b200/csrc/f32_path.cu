// fp32-accumulate draft step: every weight, activation and accumulation in
// fp32 on the CUDA cores, for checkpoints whose weights are fp32 (the CPU
// plumbing config runs mirror_sd/dflash.py on fp32 weights) and wherever the
// draft ids and accepted lengths must follow an fp32 reference exactly.
//
//   f32_gemm     C[M, N] = A[M, K] . B[N, K]^T.  Both operands stream through
//                a TMA ring (128-byte swizzle) fed by one producer warp; eight
//                consumer warps run FFMA from shared memory.  Lane l of a warp
//                owns output columns l, l+32, l+64, l+96 and reads their
//                weights as 16-byte vectors (the swizzle makes those reads
//                conflict-free); the activation values are warp-uniform
//                broadcasts.  K is split over the warps of a CTA (summed in a
//                fixed order through shared memory) and, for grid fill, over
//                CTAs into fp32 partials that f32_reduce sums in split order:
//                results do not depend on scheduling.  The lm_head variant
//                keeps only a (max, first index) per row and vocabulary tile.
//   f32_reduce   split sum + epilogue: store, residual add, or silu(g) * u
//   f32_rmsnorm  row RMSNorm (input / post-attention / hidden / final norms)
//   f32_headnorm per-head q/k RMSNorm + neox RoPE (dflash.py:290-305)
//   f32_attn     non-causal GQA attention with an fp32 online softmax over
//                [context ; block] keys (dflash.py:310-317), split over keys
//                with an ordered combine
#include <algorithm>

#include "kernels.cuh"

namespace dfl {

namespace {
__device__ __forceinline__ bool f32_better(float v, int i, float bv, int bi) {
  return (v > bv) || (v == bv && i < bi);
}
}  // namespace

constexpr int kF32BK = 64;                         // k per ring stage: two 32-float TMA boxes
constexpr int kF32BN = 128;                        // output columns (weight rows) per tile
constexpr int kF32Warps = 8;                       // consumer warps
constexpr int kF32Threads = (kF32Warps + 1) * 32;  // + the producer warp
constexpr int kF32Stages = 4;

template <int WM>
struct F32Cfg {
  static constexpr int BM = 16 * WM;               // activation rows per tile
  static constexpr int WK = kF32Warps / WM;        // warps splitting k in a CTA
  static constexpr int B_BOX = kF32BN * 128;       // 16 KB: 128 rows x 32 floats
  static constexpr int A_BOX = BM * 128;
  static constexpr int STAGE = 2 * B_BOX + 2 * A_BOX;
  static constexpr int RING = kF32Stages * STAGE;
  static constexpr int RED = kF32Warps * 16 * kF32BN * 4;  // cross-warp sums (reuses the ring)
  static constexpr int SMEM = RING + 1024 + 256;
  static_assert(RED <= RING, "reduction buffer must fit in the ring");
  static_assert(STAGE % 1024 == 0, "stage alignment");
};

// one 16-byte chunk of a 128-byte row in the TMA 128-byte swizzle
__device__ __forceinline__ const float4* f32_sw(const uint8_t* box, int row, int chunk) {
  return reinterpret_cast<const float4*>(box + row * 128 + ((chunk ^ (row & 7)) << 4));
}

// grid (n tiles, m tiles, k splits); block kF32Threads
template <int WM, bool ARGMAX>
__global__ void __launch_bounds__(kF32Threads, 1)
    f32_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const F32GemmParams p) {
  using C = F32Cfg<WM>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::RING);
  uint64_t* empty = full + kF32Stages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kF32Stages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kF32BN, m0 = blockIdx.y * C::BM;
  const int KT = p.K / kF32BK;
  const int ks0 = (int)(((long long)blockIdx.z * KT) / gridDim.z);
  const int ks1 = (int)(((long long)(blockIdx.z + 1) * KT) / gridDim.z);
  const int nsteps = ks1 - ks0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kF32Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kF32Warps);
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
  }
  __syncthreads();

  float acc[4][16];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[j][i] = 0.f;
  const int mg = warp % WM, kw = warp / WM;
  int issued = 0;   // producer: stages whose loads were issued

  if (warp == kF32Warps) {
    if (lane == 0) {
      // the weights never change: the first stages' weight boxes are issued
      // before the wait on the previous kernel, the activation boxes after it
      const int pre = min(nsteps, kF32Stages);
      for (int it = 0; it < pre; ++it) {
        uint8_t* st = smem + it * C::STAGE;
        const int kx = (ks0 + it) * kF32BK;
        mbar_arrive_expect_tx(&full[it], C::STAGE);
        tma_load_2d(st, &map_b, &full[it], kx, n0);
        tma_load_2d(st + C::B_BOX, &map_b, &full[it], kx + 32, n0);
      }
      griddep_wait();
      for (int it = 0; it < pre; ++it) {
        uint8_t* st = smem + it * C::STAGE + 2 * C::B_BOX;
        const int kx = (ks0 + it) * kF32BK;
        tma_load_2d(st, &map_a, &full[it], kx, m0);
        tma_load_2d(st + C::A_BOX, &map_a, &full[it], kx + 32, m0);
      }
      issued = pre;
      for (int it = pre; it < nsteps; ++it) {
        const int s = it % kF32Stages;
        const uint32_t ph = (it / kF32Stages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, p.err, abort_flag)) break;
        uint8_t* st = smem + s * C::STAGE;
        const int kx = (ks0 + it) * kF32BK;
        mbar_arrive_expect_tx(&full[s], C::STAGE);
        tma_load_2d(st, &map_b, &full[s], kx, n0);
        tma_load_2d(st + C::B_BOX, &map_b, &full[s], kx + 32, n0);
        tma_load_2d(st + 2 * C::B_BOX, &map_a, &full[s], kx, m0);
        tma_load_2d(st + 2 * C::B_BOX + C::A_BOX, &map_a, &full[s], kx + 32, m0);
        issued = it + 1;
      }
    }
  } else {
    for (int it = 0; it < nsteps; ++it) {
      const int s = it % kF32Stages;
      const uint32_t ph = (it / kF32Stages) & 1;
      if (!mbar_wait(&full[s], ph, p.err, abort_flag)) break;
      const uint8_t* st = smem + s * C::STAGE;
      // 16 groups of 4 k per stage; warp kw takes groups kw, kw + WK, ...
#pragma unroll 1
      for (int g = kw; g < 16; g += C::WK) {
        const uint8_t* bbox = st + (g >> 3) * C::B_BOX;
        const uint8_t* abox = st + 2 * C::B_BOX + (g >> 3) * C::A_BOX;
        const int c = g & 7;
        float4 w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = *f32_sw(bbox, lane + 32 * j, c);
#pragma unroll
        for (int iq = 0; iq < 4; ++iq) {
          float4 a[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) a[i] = *f32_sw(abox, mg * 16 + iq * 4 + i, c);
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              float t = acc[j][iq * 4 + i];
              t = fmaf(w[j].x, a[i].x, t);
              t = fmaf(w[j].y, a[i].y, t);
              t = fmaf(w[j].z, a[i].z, t);
              t = fmaf(w[j].w, a[i].w, t);
              acc[j][iq * 4 + i] = t;
            }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  // every consumer is past the ring: sum the k-warps' accumulators in order
  __syncthreads();
  if (*abort_flag) {
    // a wait gave up: let the copies still in flight land (bounded) before
    // the CTA's shared memory goes away, and write nothing
    if (warp == kF32Warps && lane == 0)
      for (int it = max(0, issued - kF32Stages); it < issued; ++it)
        for (uint32_t i = 0; i < kSpinLimit && !mbar_try_wait(&full[it % kF32Stages], (it / kF32Stages) & 1); ++i) {
        }
    return;
  }
  griddep_wait();
  griddep_launch_dependents();
  float* red = reinterpret_cast<float*>(smem);   // [WK][WM][16][128]
  if (warp < kF32Warps) {
    float* r = red + ((size_t)(kw * WM + mg) * 16) * kF32BN;
#pragma unroll
    for (int i = 0; i < 16; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) r[i * kF32BN + lane + 32 * j] = acc[j][i];
  }
  __syncthreads();
  if (!ARGMAX) {
    float* out = p.part + (size_t)blockIdx.z * p.M * p.N;
    for (int idx = threadIdx.x; idx < C::BM * kF32BN; idx += kF32Threads) {
      const int m = idx / kF32BN, n = idx % kF32BN;
      const int gm = m0 + m, gn = n0 + n;
      if (gm >= p.M || gn >= p.N) continue;
      float v = 0.f;
#pragma unroll
      for (int q = 0; q < C::WK; ++q) v += red[((size_t)(q * WM + m / 16) * 16 + m % 16) * kF32BN + n];
      out[(size_t)gm * p.N + gn] = v;
    }
  } else {
    // one warp per row: (max, first index) over this tile's columns
    for (int m = warp; m < C::BM; m += kF32Threads / 32) {
      const int gm = m0 + m;
      if (gm >= p.M) continue;
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = lane + 32 * j, gn = n0 + n;
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < C::WK; ++q) v += red[((size_t)(q * WM + m / 16) * 16 + m % 16) * kF32BN + n];
        if (gn < p.N && v == v && f32_better(v, gn, bv, bi)) { bv = v; bi = gn; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (f32_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) {
        p.best_val[(size_t)blockIdx.x * p.M + gm] = bv;
        p.best_idx[(size_t)blockIdx.x * p.M + gm] = bi;
      }
    }
  }
}

// out = sum over splits of part[s] (fixed order), then the epilogue
__global__ void f32_reduce_kernel(const float* __restrict__ part, int S, int M, int N, int mode,
                                  float* __restrict__ out, int ldo) {
  griddep_wait();
  griddep_launch_dependents();
  const int cols = mode == kF32Silu ? N / 2 : N;
  const size_t total = (size_t)M * cols;
  const size_t plane = (size_t)M * N;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(idx / cols), n = (int)(idx % cols);
    float v = 0.f;
    for (int s = 0; s < S; ++s) v += part[s * plane + (size_t)m * N + n];
    float* o = out + (size_t)m * ldo + n;
    if (mode == kF32Store) {
      *o = v;
    } else if (mode == kF32Add) {
      *o += v;
    } else {   // silu(gate) * up: gate columns [0, N/2), up columns [N/2, N)
      float u = 0.f;
      for (int s = 0; s < S; ++s) u += part[s * plane + (size_t)m * N + cols + n];
      *o = v / (1.f + expf(-v)) * u;
    }
  }
}

// y[row] = x[row] * rsqrt(mean(x[row]^2) + eps) * w (mx.fast.rms_norm); one
// CTA per row.  y2 (when given) receives rows j >= 1 of every block of
// `block` rows, packed: the lm_head's input (generate.py:604).
__global__ void f32_rmsnorm_kernel(const float* __restrict__ x, int H, const float* __restrict__ w,
                                   float eps, float* __restrict__ y, float* __restrict__ y2, int block) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float red[32];
  __shared__ float rs;
  const int row = blockIdx.x;
  const float* xr = x + (size_t)row * H;
  float ss = 0.f;
  for (int k = threadIdx.x * 4; k < H; k += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + k);
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) rs = 1.f / sqrtf(t / static_cast<float>(H) + eps);
  }
  __syncthreads();
  const float r = rs;
  const int j = row % block;
  float* y2r = (y2 && j > 0) ? y2 + ((size_t)(row / block) * (block - 1) + j - 1) * H : nullptr;
  for (int k = threadIdx.x * 4; k < H; k += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + k);
    const float4 wv = *reinterpret_cast<const float4*>(w + k);
    const float4 o = make_float4(v.x * r * wv.x, v.y * r * wv.y, v.z * r * wv.z, v.w * r * wv.w);
    if (y) *reinterpret_cast<float4*>(y + (size_t)row * H + k) = o;
    if (y2r) *reinterpret_cast<float4*>(y2r + k) = o;
  }
}

// Per-head RMSNorm (eps, learned [128] weight) and neox RoPE in place, one
// warp per (row, head): lane l holds dims 4l..4l+3, lane l ^ 16 the partner
// half.  Heads [0, nq) use wq, heads [nq, nq + nk) use wk (row r of
// layer-plane p: wk + p * 128); RoPE row = rope_row0 + r of the (cos, sin)
// table.  Rows of `planes` planes, `plane_cols` floats apart within a row.
__global__ void f32_headnorm_kernel(float* __restrict__ x, int rows, int ld, int nq, int nk, int planes,
                                    int plane_cols, const float* __restrict__ wq,
                                    const float* __restrict__ wk, const float2* __restrict__ rope,
                                    int rope_row0, float eps) {
  griddep_wait();
  griddep_launch_dependents();
  const int heads = nq + nk;
  const long long items = (long long)rows * planes * heads;
  const int lane = threadIdx.x & 31;
  for (long long it = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; it < items;
       it += ((long long)gridDim.x * blockDim.x) >> 5) {
    const int h = (int)(it % heads);
    const int pl = (int)((it / heads) % planes);
    const int r = (int)(it / ((long long)heads * planes));
    float* v = x + (size_t)r * ld + (size_t)pl * plane_cols + h * 128 + lane * 4;
    const float* w = (h < nq ? wq : wk + (size_t)pl * 128) + lane * 4;
    float4 a = *reinterpret_cast<float4*>(v);
    float ss = a.x * a.x;
    ss = fmaf(a.y, a.y, ss);
    ss = fmaf(a.z, a.z, ss);
    ss = fmaf(a.w, a.w, ss);
    ss = warp_sum(ss);
    const float rstd = 1.f / sqrtf(ss / 128.f + eps);
    const float4 wv = *reinterpret_cast<const float4*>(w);
    a = make_float4(a.x * rstd * wv.x, a.y * rstd * wv.y, a.z * rstd * wv.z, a.w * rstd * wv.w);
    float4 b;
    b.x = __shfl_xor_sync(0xffffffffu, a.x, 16);
    b.y = __shfl_xor_sync(0xffffffffu, a.y, 16);
    b.z = __shfl_xor_sync(0xffffffffu, a.z, 16);
    b.w = __shfl_xor_sync(0xffffffffu, a.w, 16);
    const float2* cs = rope + (size_t)(rope_row0 + r) * 64 + (lane & 15) * 4;
    const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 t = cs[e];   // (cos, sin) of frequency (lane & 15) * 4 + e
      // first half: x1 cos - x2 sin; second half: x1 sin + x2 cos (x1 = partner)
      o[e] = lane < 16 ? av[e] * t.x - bv[e] * t.y : bv[e] * t.y + av[e] * t.x;
    }
    *reinterpret_cast<float4*>(v) = make_float4(o[0], o[1], o[2], o[3]);
  }
}

// Attention for one (key split, q head, sequence): grid (splits, nq, nseq),
// 8 warps.  Key i of sequence s is context row ctx_start[s] + i for i < C_s,
// else block row s * block + i - C_s.  Query rows go through in passes of 16
// (2 per warp); each pass streams the split's keys in tiles of 32 through
// shared memory.  Lane l scores key l of a tile, the warp shares the max and
// sum, and lane l accumulates output dims 4l..4l+3.
constexpr int kF32AttnTile = 32;
constexpr int kF32AttnRows = 2;   // query rows per warp and pass

__global__ void __launch_bounds__(256)
    f32_attn_kernel(const F32AttnParams p) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ __align__(16) float ks[kF32AttnTile][132];
  __shared__ __align__(16) float vs[kF32AttnTile][128];
  __shared__ __align__(16) float qs[kF32Warps * kF32AttnRows][128];
  const int split = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = h / (p.nq / p.nkv);
  const int c0 = p.seq[s].ctx_start, cs = p.seq[s + 1].ctx_start - c0;
  const int n = cs + p.block;
  const int k_begin = split * p.chunk, k_end = min(n, k_begin + p.chunk);
  for (int r0 = 0; r0 < p.block; r0 += kF32Warps * kF32AttnRows) {
    // this pass's query rows
    for (int idx = threadIdx.x; idx < kF32Warps * kF32AttnRows * 32; idx += blockDim.x) {
      const int rr = idx >> 5, d4 = (idx & 31) * 4;
      const int j = r0 + rr;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (j < p.block) v = *reinterpret_cast<const float4*>(p.q + (size_t)(s * p.block + j) * p.q_ld + h * 128 + d4);
      *reinterpret_cast<float4*>(&qs[rr][d4]) = v;
    }
    float mrow[kF32AttnRows], lrow[kF32AttnRows];
    float4 acc[kF32AttnRows];
#pragma unroll
    for (int r = 0; r < kF32AttnRows; ++r) {
      mrow[r] = -INFINITY;
      lrow[r] = 0.f;
      acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int t0 = k_begin; t0 < k_end; t0 += kF32AttnTile) {
      __syncthreads();   // the previous tile (and the query rows' writes) are settled
      for (int idx = threadIdx.x; idx < kF32AttnTile * 32; idx += blockDim.x) {
        const int kr = idx >> 5, d4 = (idx & 31) * 4;
        const int i = t0 + kr;
        float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
        if (i < k_end) {
          const float* kp;
          const float* vp;
          if (i < cs) {
            kp = p.kc + (size_t)(c0 + i) * p.c_ld + hk * 128 + d4;
            vp = p.vc + (size_t)(c0 + i) * p.c_ld + hk * 128 + d4;
          } else {
            kp = p.kb + (size_t)(s * p.block + i - cs) * p.b_ld + hk * 128 + d4;
            vp = p.vb + (size_t)(s * p.block + i - cs) * p.b_ld + hk * 128 + d4;
          }
          kv = *reinterpret_cast<const float4*>(kp);
          vv = *reinterpret_cast<const float4*>(vp);
        }
        *reinterpret_cast<float4*>(&ks[kr][d4]) = kv;
        *reinterpret_cast<float4*>(&vs[kr][d4]) = vv;
      }
      __syncthreads();
      const bool valid = t0 + lane < k_end;
#pragma unroll
      for (int r = 0; r < kF32AttnRows; ++r) {
        const int rr = warp * kF32AttnRows + r;
        if (r0 + rr >= p.block) break;
        float sc = 0.f;
#pragma unroll 8
        for (int d = 0; d < 128; d += 4) {
          const float4 qv = *reinterpret_cast<const float4*>(&qs[rr][d]);
          const float4 kv = *reinterpret_cast<const float4*>(&ks[lane][d]);
          sc = fmaf(qv.x, kv.x, sc);
          sc = fmaf(qv.y, kv.y, sc);
          sc = fmaf(qv.z, kv.z, sc);
          sc = fmaf(qv.w, kv.w, sc);
        }
        sc = valid ? sc * p.scale : -INFINITY;
        const float mnew = fmaxf(mrow[r], warp_max(sc));
        const float pe = valid ? expf(sc - mnew) : 0.f;
        const float corr = expf(mrow[r] - mnew);
        lrow[r] = lrow[r] * corr + warp_sum(pe);
        mrow[r] = mnew;
        float4 a = make_float4(acc[r].x * corr, acc[r].y * corr, acc[r].z * corr, acc[r].w * corr);
#pragma unroll 8
        for (int i = 0; i < kF32AttnTile; ++i) {
          const float pi = __shfl_sync(0xffffffffu, pe, i);
          const float4 vv = *reinterpret_cast<const float4*>(&vs[i][lane * 4]);
          a.x = fmaf(pi, vv.x, a.x);
          a.y = fmaf(pi, vv.y, a.y);
          a.z = fmaf(pi, vv.z, a.z);
          a.w = fmaf(pi, vv.w, a.w);
        }
        acc[r] = a;
      }
    }
    // this split's rows: final output (one split) or (o, m, l) partials
#pragma unroll
    for (int r = 0; r < kF32AttnRows; ++r) {
      const int j = r0 + warp * kF32AttnRows + r;
      if (j >= p.block) break;
      if (p.splits == 1) {
        const float inv = 1.f / lrow[r];
        *reinterpret_cast<float4*>(p.out + (size_t)(s * p.block + j) * p.out_ld + h * 128 + lane * 4) =
            make_float4(acc[r].x * inv, acc[r].y * inv, acc[r].z * inv, acc[r].w * inv);
      } else {
        const size_t prow = (((size_t)s * p.nq + h) * p.splits + split) * p.block + j;
        *reinterpret_cast<float4*>(p.opart + prow * 128 + lane * 4) = acc[r];
        if (lane == 0) {
          p.mpart[prow] = mrow[r];
          p.lpart[prow] = lrow[r];
        }
      }
    }
  }
}

// merge the key splits of every (sequence, head, row) in split order; one warp each
__global__ void f32_attn_combine_kernel(const F32AttnParams p) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const long long items = (long long)p.nseq * p.nq * p.block;
  for (long long it = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; it < items;
       it += ((long long)gridDim.x * blockDim.x) >> 5) {
    const int j = (int)(it % p.block);
    const int h = (int)((it / p.block) % p.nq);
    const int s = (int)(it / ((long long)p.block * p.nq));
    const size_t base = (((size_t)s * p.nq + h) * p.splits) * p.block + j;
    float mx = -INFINITY;
    for (int q = 0; q < p.splits; ++q) mx = fmaxf(mx, p.mpart[base + (size_t)q * p.block]);
    float l = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < p.splits; ++q) {
      const size_t pr = base + (size_t)q * p.block;
      const float m = p.mpart[pr];
      if (m == -INFINITY) continue;   // a split with no keys of this sequence
      const float f = expf(m - mx);
      l = fmaf(p.lpart[pr], f, l);
      const float4 v = *reinterpret_cast<const float4*>(p.opart + pr * 128 + lane * 4);
      o.x = fmaf(v.x, f, o.x);
      o.y = fmaf(v.y, f, o.y);
      o.z = fmaf(v.z, f, o.z);
      o.w = fmaf(v.w, f, o.w);
    }
    const float inv = 1.f / l;
    *reinterpret_cast<float4*>(p.out + (size_t)(s * p.block + j) * p.out_ld + h * 128 + lane * 4) =
        make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
  }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFnF)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// fp32 [rows, K] row-major, boxes of 32 floats x box_rows in the 128-byte swizzle
static bool f32_map(CUtensorMap* m, const float* base, uint64_t K, uint64_t rows, uint32_t box_rows) {
  static EncodeTiledFnF fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return false;
    fn = reinterpret_cast<EncodeTiledFnF>(ptr);
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (K * 4) % 16) return false;
  cuuint64_t dims[2] = {K, rows};
  cuuint64_t strides[1] = {K * 4};
  cuuint32_t box[2] = {32, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int f32_wm(int M) { return M <= 16 ? 1 : (M <= 32 ? 2 : 4); }

// k splits: minimise the makespan in k-step units, waves * (steps per split
// + a fixed cost of 2 steps per CTA), within the partial buffer
int f32_gemm_splits(int M, int N, int K, int num_sms, size_t part_floats) {
  const int BM = 16 * f32_wm(M);
  const long long tiles = (long long)((N + kF32BN - 1) / kF32BN) * ((M + BM - 1) / BM);
  const int KT = K / kF32BK;
  int best = 1;
  double best_cost = 1e30;
  for (int S = 1; S <= std::min(32, std::max(1, KT / 2)); ++S) {
    if ((size_t)S * M * N > part_floats) break;
    const long long ctas = tiles * S;
    const double waves = (double)((ctas + num_sms - 1) / num_sms);
    const double cost = waves * ((double)KT / S + 2.0);
    if (cost < best_cost * 0.98) {
      best_cost = cost;
      best = S;
    }
  }
  return best;
}

template <int WM, bool ARGMAX>
static cudaError_t f32_gemm_go(const CUtensorMap& ma, const CUtensorMap& mb, const F32GemmParams& p, int S,
                               cudaStream_t st) {
  using C = F32Cfg<WM>;
  auto kern = f32_gemm_kernel<WM, ARGMAX>;
  DFL_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
  DFL_TRY(max_smem_carveout(kern));
  dim3 grid((p.N + kF32BN - 1) / kF32BN, (p.M + C::BM - 1) / C::BM, S);
  return launch_pdl(kern, grid, dim3(kF32Threads), (size_t)C::SMEM, st, ma, mb, p);
}

cudaError_t f32_gemm_launch(const float* A, const float* B, int mode, F32GemmParams p, float* out, int ldo,
                            int num_sms, cudaStream_t st) {
  if (p.M < 1 || p.N < 1 || p.K < kF32BK || p.K % kF32BK) return cudaErrorInvalidValue;
  const int wm = f32_wm(p.M);
  CUtensorMap ma, mb;
  if (!f32_map(&ma, A, p.K, p.M, 16 * wm) || !f32_map(&mb, B, p.K, p.N, kF32BN)) return cudaErrorInvalidValue;
  if (mode == kF32Argmax) {
    if (!p.best_val || !p.best_idx) return cudaErrorInvalidValue;
    switch (wm) {
      case 1: return f32_gemm_go<1, true>(ma, mb, p, 1, st);
      case 2: return f32_gemm_go<2, true>(ma, mb, p, 1, st);
      default: return f32_gemm_go<4, true>(ma, mb, p, 1, st);
    }
  }
  if (!p.part || (mode == kF32Silu && p.N % 2)) return cudaErrorInvalidValue;
  const int S = f32_gemm_splits(p.M, p.N, p.K, num_sms, p.part_floats);
  if ((size_t)S * p.M * p.N > p.part_floats) return cudaErrorInvalidValue;
  cudaError_t e;
  switch (wm) {
    case 1: e = f32_gemm_go<1, false>(ma, mb, p, S, st); break;
    case 2: e = f32_gemm_go<2, false>(ma, mb, p, S, st); break;
    default: e = f32_gemm_go<4, false>(ma, mb, p, S, st); break;
  }
  DFL_TRY(e);
  DFL_TRY(max_smem_carveout(f32_reduce_kernel));
  const size_t total = (size_t)p.M * (mode == kF32Silu ? p.N / 2 : p.N);
  const int blocks = (int)std::min<size_t>((total + 255) / 256, (size_t)num_sms * 8);
  return launch_pdl(f32_reduce_kernel, dim3(std::max(blocks, 1)), dim3(256), 0, st, (const float*)p.part, S,
                    p.M, p.N, mode, out, ldo);
}

cudaError_t f32_rmsnorm_launch(const float* x, int rows, int H, const float* w, float eps, float* y, float* y2,
                               int block, cudaStream_t st) {
  if (rows < 1) return cudaSuccess;
  if (H % 4 || block < 1 || (y2 && rows % block)) return cudaErrorInvalidValue;
  DFL_TRY(max_smem_carveout(f32_rmsnorm_kernel));
  return launch_pdl(f32_rmsnorm_kernel, dim3(rows), dim3(256), 0, st, x, H, w, eps, y, y2, block);
}

cudaError_t f32_headnorm_launch(float* x, int rows, int ld, int nq, int nk, int planes, int plane_cols,
                                const float* wq, const float* wk, const float2* rope, int rope_row0, float eps,
                                int num_sms, cudaStream_t st) {
  if (rows < 1) return cudaSuccess;
  DFL_TRY(max_smem_carveout(f32_headnorm_kernel));
  const long long warps = (long long)rows * planes * (nq + nk);
  const int blocks = (int)std::min<long long>((warps + 7) / 8, (long long)num_sms * 16);
  return launch_pdl(f32_headnorm_kernel, dim3(blocks), dim3(256), 0, st, x, rows, ld, nq, nk, planes, plane_cols,
                    wq, wk, rope, rope_row0, eps);
}

void f32_attn_pick_split(int nseq, int nq, int kv_len_max, int num_sms, int max_splits, int* chunk, int* splits) {
  const int tiles = std::max(1, (kv_len_max + kF32AttnTile - 1) / kF32AttnTile);
  int s = std::max(1, (2 * num_sms + nseq * nq - 1) / (nseq * nq));
  s = std::min(std::min(s, tiles), max_splits);
  const int per = (tiles + s - 1) / s;
  *chunk = per * kF32AttnTile;
  *splits = (tiles + per - 1) / per;
}

cudaError_t f32_attn_launch(const F32AttnParams& p, int num_sms, cudaStream_t st) {
  if (p.nkv < 1 || p.nq % p.nkv || p.block < 1 || p.splits < 1) return cudaErrorInvalidValue;
  DFL_TRY(max_smem_carveout(f32_attn_kernel));
  DFL_TRY(launch_pdl(f32_attn_kernel, dim3(p.splits, p.nq, p.nseq), dim3(256), 0, st, p));
  if (p.splits == 1) return cudaSuccess;
  DFL_TRY(max_smem_carveout(f32_attn_combine_kernel));
  const long long warps = (long long)p.nseq * p.nq * p.block;
  const int blocks = (int)std::min<long long>((warps + 7) / 8, (long long)num_sms * 16);
  return launch_pdl(f32_attn_combine_kernel, dim3(blocks), dim3(256), 0, st, p);
}

}  // namespace dfl
