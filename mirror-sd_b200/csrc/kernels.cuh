// Host/device parameter blocks and host launch functions of every kernel.
#pragma once
#include "w8_gemm.cuh"

namespace dfl {

struct AttnParams {
  const __half* q;      // [b, NQ, B, 128]
  const __half* k;      // [b, NKV, kv_cap, 128]
  const __half* v;      // [b, NKV, kv_cap, 128]
  int nq, nkv, block, kv_len, kv_cap;
  int chunk, splits;    // kv rows per CTA (multiple of 64), CTAs per (b, kv head)
  float* opart;         // [b, NKV, splits, R, 128]
  float* mpart;         // [b, NKV, splits, R]  (base-2 logits)
  float* lpart;
  float scale_log2;     // head_dim^-0.5 * log2(e)
  int normrope;
  const float* q_norm;
  const float* k_norm;
  const float2* rope;   // [rows, 64] (cos, sin) table
  float eps;
  int q_row0, k_row0;   // table rows: q row j -> q_row0 + j, k row i -> k_row0 + i
};

enum TcMode : int { kTcFc = 0, kTcCtxKV = 1, kTcStoreF32 = 2 };

struct TcParams {
  int M, N, K;
  int* err;
  // kTcFc and kTcStoreF32
  float* out_f32;           // [M, N]
  float* sumsq_part;        // kTcFc: [N/256, M] partial sums of squares per row
  // kTcCtxKV
  const float* scale;       // [N]
  const float* k_norm;      // [L, 128]
  const float2* rope;       // [rows, 64] (cos, sin) by kv row
  __half* k_out;            // layer l base = k_out + l * layer_stride
  __half* v_out;
  size_t layer_stride;      // halves
  int nkv, rows_per_seq, kv_cap, kv_row0;
  float eps;
};

struct LmParams {
  const __nv_bfloat16* E;   // [V, H]
  const __nv_bfloat16* hn;  // [M, H]
  int V, H, M;
  float* best_val;          // [gridDim.x, M]
  int* best_idx;
};

// ---- host launchers (return cudaErrorInvalidValue on unsupported shapes)
cudaError_t w8_gemm_launch(const W8Params& p, int mode, cudaStream_t st);
cudaError_t rmsnorm_f16_launch(const float* h, const float* hstat, int hparts, int M, int K,
                               const float* w, float eps, __half* x, cudaStream_t st);
int w8_pick_splits(int N, int K, int M, int num_sms, int max_splits);
// tcgen05 W8A16 path (w8_tc.cu): w_tiles is the int8 weight packed by
// w8_tilepack_launch ([N/128][K/64][128][64 B]); part / counters are the
// split-K scratch (w8tc_part_floats floats; counters zero, one per tile).
void w8tc_plan(int N, int K, int num_sms, int* splits, int* groups);
size_t w8tc_part_floats(int N, int K, int M, int num_sms);
cudaError_t w8tc_launch(const int8_t* w_tiles, const W8Params& p, int mode, int* err, float* part,
                        size_t part_floats, int* counters, int num_sms, cudaStream_t st);
cudaError_t w8_tilepack_launch(const int8_t* src, int n_src, int K, int8_t* dst, int grp, int gstride,
                               int base, cudaStream_t st);
size_t w8_smem_bytes(const W8Params& p);
cudaError_t w8_repack_launch(const int8_t* src, int n_src, int K, uint8_t* dst, int grp,
                             int gstride, int base, cudaStream_t st);
cudaError_t w8_scale_launch(const __half* s, int n_src, float* dst, int grp, int gstride,
                            int base, cudaStream_t st);
cudaError_t quantize_q8_launch(const float* w, int oc, int ic, int8_t* q, __half* s,
                               cudaStream_t st);

size_t attn_smem_bytes(int nq, int nkv, int block);
void attn_pick_split(int batch, int nkv, int kv_len, int num_sms, int* chunk, int* splits);
cudaError_t attn_launch(const AttnParams& p, int batch, __half* out, cudaStream_t st);

cudaError_t tc_gemm_launch(const void* A, const void* B, bool bf16, int mode, const TcParams& p,
                           cudaStream_t st);

int lm_grid(int V, int num_sms);
size_t lm_pack_bytes(int V, int H);
cudaError_t lm_pack_launch(const __nv_bfloat16* E, int V, int H, uint8_t* out, cudaStream_t st);
cudaError_t lm_argmax_launch(const LmParams& p, const uint8_t* e_tiles, int num_sms, int* err,
                             int* grid_out, cudaStream_t st);
cudaError_t argmax_accept_launch(const float* bv, const int* bi, int nparts, int M, int block,
                                 int batch, int32_t* out_tokens, const int32_t* target,
                                 int32_t* acc_len, int32_t* correction, cudaStream_t st);
cudaError_t accept_launch(const int32_t* draft, const int32_t* target, int batch, int block,
                          int32_t* acc_len, int32_t* correction, cudaStream_t st);

cudaError_t rope_table_launch(int pos0, int rows, const float* inv_freq, float2* out, cudaStream_t st);
cudaError_t init_h_launch(const __nv_bfloat16* noise, int M, int H, float* h, float* hstat,
                          cudaStream_t st);
cudaError_t ctx_norm_launch(const float* raw, const float* part, int nparts, int rows, int H,
                            const float* w, float eps, __half* out, cudaStream_t st);
cudaError_t final_norm_launch(const float* h, const float* hstat, int hparts, int M, int H,
                              const float* w, float eps, __nv_bfloat16* hn, void* out, bool out_f32,
                              cudaStream_t st);
cudaError_t i8_to_f16_launch(const int8_t* src, size_t n, __half* dst, cudaStream_t st);
cudaError_t f16_to_f32_launch(const __half* src, size_t n, float* dst, cudaStream_t st);

}  // namespace dfl
