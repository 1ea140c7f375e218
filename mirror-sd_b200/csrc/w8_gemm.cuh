// W8A16 skinny GEMM for the block rows of the DFlash draft forward.
//
//   Y[m, n] = scale[n] * sum_k X[m, k] * Wq[n, k]        (m < M <= 64 rows)
//
// Wq is the reference's int8 per-output-channel weight (ane_model.py:265-279)
// repacked once at load time (w8_repack) so that every 128-channel tile is one
// contiguous run of 8 KB k64-blocks and each warp streams its own 2 KB of every
// block with four fully coalesced 512-byte loads; the bytes are stored biased
// (q + 128) so a single PRMT against 0x6464 builds the f16 value 1024 + u and
// one f16x2 subtract recovers q exactly.  Weights are prefetched straight into
// registers several k-blocks ahead; the f16 activations stream through a
// shared-memory ring (cp.async) shared by the CTA's four warps.  The MMA runs
// swap-AB on mma.sync m16n8k16 (16 output channels x 8 activation rows per
// op), fp32 accumulate.
//
// K is split across the CTAs of a thread-block cluster (at most 8, portable);
// partial tiles are reduced through distributed shared memory in a fixed rank
// order (deterministic, no global scratch), then a fused epilogue runs:
//   kStore   : Y as f16
//   kQKV     : per-head RMSNorm + neox RoPE for q and k heads, plain v, written
//              into the attention layouts (dflash.py:290-305)
//   kResid   : h += Y (fp32 residual stream) and per-128-channel sum of h^2
//              partials for the next RMSNorm (dflash.py:356, :361)
//   kSiluMul : each 128-channel tile holds 64 gate and the 64 matching up
//              channels -> silu(g) * u (dflash.py:330)
#pragma once
#include "common.cuh"

namespace dfl {

enum W8Mode : int { kStore = 0, kQKV = 1, kResid = 2, kSiluMul = 3 };

constexpr int W8_WARPS = 4;
constexpr int W8_NT = W8_WARPS * 32;  // output channels per CTA tile
constexpr int W8_PD = 4;              // k64 weight blocks in flight per warp
constexpr int W8_CHK = 256;           // activation k per ring stage
constexpr int W8_NST = 3;             // ring stages
constexpr int W8_XLD = W8_CHK + 8;    // halves per staged row (+16 B keeps reads conflict free)

struct W8Params {
  const uint8_t* w;       // packed biased weights, N x K
  const float* scale;     // [N] fp32 per-output-channel scale (from the fp16 scale)
  int N, K, M;            // M = activation rows (batch * block)
  int splits;             // cluster size along K
  const __half* x;        // [M, K] f16 activations
  // outputs
  __half* y;              // kStore: [M, N]
  float* h_out;           // kResid: [M, N] (in place residual)
  float* hstat_out;       // kResid: [N/128, M]
  __half* act;            // kSiluMul: [M, N/2]
  // kQKV
  __half* q_out;          // [b, NQ, B, 128]
  __half* k_out;          // [b, NKV, kv_rows, 128], block rows start at kv_row0
  __half* v_out;
  const float* q_norm;    // [128]
  const float* k_norm;    // [128]
  const float2* rope;     // [kv rows, 64] (cos, sin); q and block-k rows use kv_row0 + j
  float eps;
  int n_q_heads, n_kv_heads, block, kv_rows, kv_row0;
};

// Packed layout: for tile t in N/128, kb in K/64: 8 KB; inside it warp w
// (channels t*128 + 32w .. +31) owns 2 KB = [rb 2][half 2][lane 32][16 B];
// lane = 4*g + c; half 0 holds row 16*rb + g of the warp, half 1 row +8;
// byte j is W[row][kb*64 + 16*c + j] + 128.
__host__ __device__ inline size_t w8_packed_offset(int tile, int kb, int warp, int rb, int half,
                                                   int lane, int K) {
  return (((((size_t)tile * (K / 64) + kb) * W8_WARPS + warp) * 2 + rb) * 2 + half) * 512 +
         (size_t)lane * 16;
}

}  // namespace dfl
