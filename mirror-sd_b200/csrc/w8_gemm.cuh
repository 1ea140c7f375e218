// W8A16 skinny GEMM for the block rows of the DFlash draft forward.
//
//   Y[m, n] = scale[n] * sum_k X[m, k] * Wq[n, k]        (m < M <= 64 rows)
//
// Wq is the reference's int8 per-output-channel weight (ane_model.py:265-279)
// repacked once at load time (w8_repack) so that one 128-bit load per lane
// yields the int8 operands of four m16n8k16 MMAs; the bytes are stored biased
// (q + 128) so a single PRMT against 0x6464 builds the f16 value 1024 + u and
// one f16x2 subtract recovers q exactly.  X (f16) sits in shared memory.  The
// MMA runs swap-AB (weights are the 16-row A operand, the <= 64 activation
// rows are N), so the tensor core is fed 16 output channels x 8 rows per op.
// K is split across the CTAs of a thread-block cluster; partial tiles are
// reduced through distributed shared memory in a fixed rank order
// (deterministic, no global scratch), then a fused epilogue runs:
//   kStore   : Y as f16
//   kQKV     : per-head RMSNorm + neox RoPE for q and k heads, plain v, written
//              into the attention layouts (dflash.py:290-305)
//   kResid   : h += Y (fp32 residual stream) and per-128-channel sum of h^2
//              partials for the next RMSNorm (dflash.py:356, :361)
//   kSiluMul : gate/up interleaved per 256-channel tile -> silu(g) * u (:330)
#pragma once
#include "common.cuh"

namespace dfl {

enum W8Mode : int { kStore = 0, kQKV = 1, kResid = 2, kSiluMul = 3 };
enum W8XSrc : int { kXF16 = 0, kXHNorm = 1 };

constexpr int W8_WARPS = 8;
constexpr int W8_NT = W8_WARPS * 32;  // output channels per CTA tile
constexpr int W8_PD = 4;              // k64 blocks kept in flight per warp

struct W8Params {
  const uint8_t* w;       // packed biased weights, N x K
  const float* scale;     // [N] fp32 per-output-channel scale (from the fp16 scale)
  int N, K, M;            // M = activation rows (batch * block)
  int splits;             // cluster size along K
  // activation source
  const __half* x;        // kXF16: [M, K]
  const float* h;         // kXHNorm: [M, K] fp32 residual stream
  const float* hstat;     // kXHNorm: [hparts, M] partial sums of h^2
  int hparts;
  const float* norm_w;    // kXHNorm: [K] RMSNorm weight
  float eps;
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
  int n_q_heads, n_kv_heads, block, kv_rows, kv_row0;
  int* err;
};

// Packed layout: for rb in N/16, kb in K/64, half in {0,1}, lane in 32: 16 bytes.
// lane = 4*g + c; half 0 holds row rb*16+g, half 1 row rb*16+g+8; byte j is
// W[row][kb*64 + 16*c + j] + 128.
__host__ __device__ inline size_t w8_packed_offset(int rb, int kb, int half, int lane, int K) {
  return ((((size_t)rb * (K / 64) + kb) * 2 + half) * 32 + lane) * 16;
}

}  // namespace dfl
