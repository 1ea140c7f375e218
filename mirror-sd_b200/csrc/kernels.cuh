// Host/device parameter blocks and host launch functions of every kernel.
#pragma once
#include "common.cuh"

namespace dfl {

// ---- where K/V rows live ----------------------------------------------------
//
// Every K/V store is [layer][sequence][kv head][slots][128] f16.  A sequence's
// stored rows form the logical list of the reference cache
// (dflash.py:139-212): the first `sink` logical rows sit in slots [0, sink);
// the rest live in a ring of `ring` slots after them, logical row p >= sink
// at slot sink + (rs + p - sink) mod ring.  Eviction of the middle rows moves
// the ring start `rs` only, trim shortens the list: no K/V row is ever copied.
// The stateless forward (cache=None) is the case sink = 0, rs = 0, n0 = 0.
//
// One forward appends each sequence's new context rows and then its block
// rows; appended row i of sequence s is logical row n0[s] + i, at RoPE
// position pos0[s] + i.  Context rows are packed across sequences
// ([ctx_start[s], ctx_start[s+1]) in the fc / context GEMMs); the RoPE table
// holds the packed context rows first and then the nseq * block block rows.
// Per-sequence record of one forward (host-built, device-resident).
struct KvSeq {
  int ctx_start;   // first packed context row of the sequence (entry nseq: total rows)
  int n0;          // logical rows stored before this forward
  int rs_pre;      // ring start while appending
  int rs_post;     // ring start after eviction (what attention reads)
  int n_att;       // logical rows attention reads
  int pos0;        // RoPE position of appended row 0
  int cseq;        // the sequence's index in the K/V store (its cache slot)
};

struct KvMap {
  int nseq;                        // 0: plain [seq][kv head][slots] layout, rows 0..kv_len-1
  int sink, ring, slots;           // slots = sink + ring
  const KvSeq* seq;                // device [nseq + 1]; read only after griddep_wait
};

// the records travel to the device as a kernel parameter of the first kernel
// of a forward (rope_table_map) or, beyond kKvChunk records, of kv_upload
// launches before it
constexpr int kKvChunk = 150;
struct KvUpload {
  int n, off;                      // records [off, off + n) of the map
  KvSeq s[kKvChunk];
};

__host__ __device__ __forceinline__ int kv_slot(const KvMap& m, int p, int rs) {
  if (p < m.sink) return p;
  int j = rs + (p - m.sink);
  if (j >= m.ring) j -= m.ring;
  return m.sink + j;
}

// sequence owning packed context row `row` (the last s with seq[s].ctx_start <= row)
__host__ __device__ __forceinline__ int kv_seq_of_ctx_row(const KvSeq* seq, int nseq, int row) {
  int lo = 0, hi = nseq - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (seq[mid].ctx_start <= row) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// W8A16 projections (w8_tc.cu).  Activations enter as three int8 limbs per
// element with a power-of-two scale per row (w8_limbs / rmsnorm_limbs):
// int8 [3][MP][K] limb-major, MP = M padded to 16, rows >= M zero.
// Epilogues:
//   kStore   : Y as f16
//   kQKV     : per-head RMSNorm + neox RoPE for q and k heads, plain v, written
//              into the attention layouts (dflash.py:290-305)
//   kResid   : h += Y (fp32 residual stream) and per-128-channel sum of h^2
//              partials for the next RMSNorm (dflash.py:356, :361)
//   kSiluMul : each 128-channel tile holds 64 gate and the 64 matching up
//              channels -> silu(g) * u (dflash.py:330)
enum W8Mode : int { kStore = 0, kQKV = 1, kResid = 2, kSiluMul = 3 };

struct W8Params {
  const float* scale;     // [N] fp32 per-output-channel scale (from the fp16 scale)
  int N, K, M;            // M = activation rows (batch * block)
  int splits;             // grid size (set by w8tc_launch)
  const int8_t* xl;       // activation limbs [3][MP][K]
  const float* xscale;    // [MP] row scales (powers of two)
  // outputs
  __half* y;              // kStore: [M, N]
  float* h_out;           // kResid: [M, N] (in place residual)
  float* hstat_out;       // kResid: [N/128, M] partial sums of h^2
  float* hmax_out;        // kResid: [N/128, M] partial max |h * next_norm| (or NULL)
  const float* next_norm; // kResid: weight of the RMSNorm that reads h next
  float* act;             // kSiluMul: [M, N/2] fp32 (no f16 range limit before the limb split)
  float* amax_out;        // kSiluMul: [N/128, M] partial max |act| (or NULL)
  // kQKV
  __half* q_out;          // [b, NQ, B, 128]
  __half* k_out;          // this layer's K store [seq][NKV][kv.slots][128] (KvMap)
  __half* v_out;
  const float* q_norm;    // [128]
  const float* k_norm;    // [128]
  const float2* rope;     // (cos, sin) table; block row m = s * block + j uses row rope_blk0 + m
  float eps;
  int n_q_heads, n_kv_heads, block, rope_blk0;
  KvMap kv;               // block row j of sequence s is logical row n0[s] + ctx_s + j
};

struct AttnParams {
  const __half* q;      // [b, NQ, B, 128]
  const __half* k;      // [b, NKV, kv_cap, 128] (kv_cap = kv.slots when kv.nseq > 0)
  const __half* v;
  int nq, nkv, block, kv_len, kv_cap;  // kv_len: longest logical row count
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
  KvMap kv;             // nseq > 0: sequence s reads logical rows [0, n_att[s]) at rs_post[s]
                        // of K/V store sequence cseq[s]
  int kv_seqs;          // nseq > 0: sequences in the K/V store (k, v hold kv_seqs * NKV planes)
  float* omax;          // combine: [NQ, b * block] max |out| per head and row (or NULL)
  __half* out;          // tcgen05 kernel with one split: the final rows, written directly
                        // (no partials, no combine); set by attn_tc_launch
  int* err;             // device error word for bounded waits (tcgen05 kernel), or NULL
};

// Persistent tcgen05 GEMM epilogues (tc_gemm.cu).  The last four serve the
// block rows once batch * block is a dense contraction (above the W8A16
// kernel's 64 rows): weights as exact f16 copies of the int8 values, the
// per-channel scale applied here.
//   kTcFc     : fp32 store + per-256-column sums of squares (hidden_norm input)
//   kTcCtxKV  : context K | V of every layer: scale, k RMSNorm + RoPE, KvMap slots
//   kTcStoreF32 : plain fp32 store
//   kTcBlkQKV : block q | k | v heads: scale, q/k RMSNorm + RoPE, q -> q_out,
//               k / v -> KvMap slots (dflash.py:290-305)
//   kTcResid  : h += acc * scale, per-256-column sums of h^2 (dflash.py:356, :361)
//   kTcSilu   : 128 gate then 128 up columns per tile -> silu(g) * u (dflash.py:330)
//   kTcArgmax : B = lm_head vocabulary tiles (lm_pack layout); per-tile row
//               argmax partials (generate.py:604-606)
enum TcMode : int { kTcFc = 0, kTcCtxKV = 1, kTcStoreF32 = 2, kTcBlkQKV = 3, kTcResid = 4, kTcSilu = 5,
                    kTcArgmax = 6 };

struct TcParams {
  int M, N, K;
  int a_cols;               // K columns per A source (tc_gemm_launch_src); K for one source
  int* err;
  // tail split (set by the launcher): the partial last round of tiles is cut
  // along K into `split` parts; workspace tail_part [tail_cap][128 * 256]
  // fp32, tail_cnt [SMs] zero between launches.  NULL workspace: no split.
  float* tail_part;
  int* tail_cnt;
  int tail_cap;             // partial slots of 128 * 256 floats in tail_part
  int split;
  // kTcFc and kTcStoreF32
  float* out_f32;           // [M, N]
  float* sumsq_part;        // kTcFc: [N/256, M] partial sums of squares per row
  // kTcFc with out_b16: bf16(acc * colw[col]) instead of the fp32 store (the
  // fc output times the hidden_norm weight, in the reference's activation
  // type so an unnormalised row cannot overflow; the row's 1/rms is applied
  // by the GEMM that reads it, kTcCtxKV with row_sumsq)
  __nv_bfloat16* out_b16;
  const float* colw;
  // kTcCtxKV: when set, rows are scaled by rsqrt(sum_q row_sumsq[q, row] / row_dim + eps)
  const float* row_sumsq;   // [row_parts, M]
  int row_parts, row_dim;
  // kTcCtxKV
  const float* scale;       // [N]
  const float* k_norm;      // [L, 128]
  const float2* rope;       // (cos, sin) table, row = packed context row
  __half* k_out;            // layer l base = k_out + l * layer_stride, [seq][NKV][kv.slots][128]
  __half* v_out;
  size_t layer_stride;      // halves
  int nkv;
  float eps;
  KvMap kv;                 // packed context row -> (sequence, logical row, slot)
  // kTcBlkQKV (k_out / v_out: this layer's store, k_norm: this layer's [128])
  __half* q_out;            // [b, NQ, block, 128]
  const float* q_norm;      // [128]
  int n_q_heads, block, rope_row0;   // block row m uses table row rope_row0 + m
  // kTcResid (sumsq_part: [N/256, M])
  float* h;                 // [M, N] residual stream, updated in place
  // kTcSilu
  __half* act;              // [M, N/2]
  // kTcArgmax
  int V;                    // vocabulary size (columns >= V are ignored)
  float* best_val;          // [N/256, M]
  int* best_idx;
};

struct LmParams {
  const __nv_bfloat16* E;   // [V, H]
  const __nv_bfloat16* hn;  // [M, H]
  int V, H, M;
  float* best_val;          // [gridDim.x, M]
  int* best_idx;
};

// ---- host launchers (return cudaErrorInvalidValue on unsupported shapes)
// tcgen05 W8A16 path (w8_tc.cu): w_tiles is the int8 weight packed by
// w8_tilepack_launch ([N/128][K/128][128][128 B], swizzled); part / counters
// are the split-K scratch (w8tc_part_floats floats; counters zero, one per tile).
// maxpart: [nparts, M] partial row maxima of |x| from the producer (or NULL:
// the kernel finds the maxima itself, one CTA per row)
cudaError_t w8_limbs_launch(const __half* x, int M, int K, const float* maxpart, int nparts,
                            int8_t* xl, float* xscale, cudaStream_t st);
cudaError_t w8_limbs_launch(const float* x, int M, int K, const float* maxpart, int nparts,
                            int8_t* xl, float* xscale, cudaStream_t st);
// x = h * rsqrt(mean h^2 + eps) * w (fp32) -> limbs; hstat / hmax: [hparts, M]
// partial sums of h^2 and partial maxima of |h * w|
cudaError_t rmsnorm_limbs_launch(const float* h, const float* hstat, const float* hmax, int hparts,
                                 int M, int K, const float* w, float eps, int8_t* xl, float* xscale,
                                 cudaStream_t st);
size_t w8tc_part_floats(int N, int K, int M, int num_sms);
cudaError_t w8tc_launch(const int8_t* w_tiles, const W8Params& p, int mode, int* err, float* part,
                        size_t part_floats, int* counters, int num_sms, cudaStream_t st);
cudaError_t w8_tilepack_launch(const int8_t* src, int n_src, int K, int8_t* dst, int grp, int gstride,
                               int base, cudaStream_t st);
cudaError_t w8_scale_launch(const __half* s, int n_src, float* dst, int grp, int gstride,
                            int base, cudaStream_t st);
cudaError_t quantize_q8_launch(const float* w, int oc, int ic, int8_t* q, __half* s,
                               cudaStream_t st);

size_t attn_smem_bytes(int nq, int nkv, int block);
// rows: query rows per kv head (heads / kv heads * block)
void attn_pick_split(int batch, int nkv, int kv_len, int num_sms, int rows, int* chunk, int* splits);
int attn_max_splits(int batch, int nkv, int num_sms, int rows);
// mma.sync split kernel (also the fused QK-norm + RoPE variant) + combine
cudaError_t attn_launch(const AttnParams& p, int batch, __half* out, cudaStream_t st);
// The o-projection's input as W8A16 limbs ([3][MP][NQ*128] limb-major, MP =
// M padded to 16, rows >= M zero; power-of-two row scales), written by the
// split merge when it can (more than one KV split, at most 64 query heads):
// attn_tc_launch then sets `done` and writes no f16 rows.
struct AttnLimbOut {
  int8_t* xl;
  float* xscale;
  int M;       // activation rows (batch * block)
  bool done;
};
// tcgen05 split kernel (S and O in TMEM; no normrope) + combine
cudaError_t attn_tc_launch(const AttnParams& p, int batch, __half* out, cudaStream_t st,
                           AttnLimbOut* limbs = nullptr);
cudaError_t attn_combine_launch(const AttnParams& p, int batch, __half* out, cudaStream_t st);
cudaError_t attn_combine_limbs_launch(const AttnParams& p, int batch, const AttnLimbOut& lo, cudaStream_t st);

// A given as column blocks held in separate arrays: A[:, f*cols:(f+1)*cols] is
// ptr[f] (rows ld[f] elements apart), f < n; n * cols == K
constexpr int kTcMaxSrc = 8;
struct TcSources {
  const void* ptr[kTcMaxSrc];
  long long ld[kTcMaxSrc];
  int n;
  int cols;
};
cudaError_t tc_gemm_launch_src(const TcSources& a, const void* B, bool bf16, int mode, TcParams p,
                               cudaStream_t st);
cudaError_t tc_gemm_launch(const void* A, const void* B, bool bf16, int mode, const TcParams& p,
                           cudaStream_t st);

int lm_grid(int V, int num_sms);
size_t lm_pack_bytes(int V, int H);
cudaError_t lm_pack_launch(const __nv_bfloat16* E, int V, int H, uint8_t* out, cudaStream_t st);
cudaError_t lm_argmax_launch(const LmParams& p, const uint8_t* e_tiles, int num_sms, int* err,
                             int* grid_out, cudaStream_t st);
// per-row argmax partials [nparts, M] -> draft ids of rows 1..block-1 and
// acceptance; first = 1 when the partial rows omit row 0 of every block
// (M = batch * (block - 1))
cudaError_t argmax_accept_launch(const float* bv, const int* bi, int nparts, int M, int block,
                                 int batch, int32_t* out_tokens, const int32_t* target,
                                 int32_t* acc_len, int32_t* correction, cudaStream_t st, int first = 0);
cudaError_t accept_launch(const int32_t* draft, const int32_t* target, int batch, int block,
                          int32_t* acc_len, int32_t* correction, cudaStream_t st);

// soft anchor (anchor.cu): rows of logits -> bf16 weighted embedding rows
constexpr int kSaMaxK = 16;        // top-k bound
constexpr int kSaMaxCtas = 160;    // CTAs per row bound (candidate workspace)
struct SaParams {
  const void* logits;   // [rows, ld] fp32, or bf16 when logits_bf16
  int logits_bf16;
  int V;
  long long ld;         // elements between rows of logits
  int k;
  const void* E;        // bf16 [V, H] row-major, or lm_pack tiles
  int H;
  __nv_bfloat16* out;   // [rows, out_ld]
  long long out_ld;
  float* cand_v;        // [rows, kSaMaxCtas, kSaMaxK]
  int* cand_i;
  int* counter;         // [rows], zero between launches
};
int soft_anchor_ctas(int V, int rows, int num_sms);
cudaError_t soft_anchor_launch(const SaParams& p, int rows, bool e_tiled, int num_sms, cudaStream_t st);
// (cos, sin) rows for positions pos0 .. pos0 + rows - 1, inv_freq from theta on the device
cudaError_t rope_table_launch(int pos0, int rows, float theta, float2* out, cudaStream_t st);
// table rows of one forward: packed context rows, then nseq * block block rows.
// Also stores the map's records (host array `seq`, nseq + 1 entries) at m.seq.
cudaError_t rope_table_map_launch(const KvMap& m, const KvSeq* seq, int block, const float* inv_freq,
                                  float2* out, cudaStream_t st);
cudaError_t init_h_launch(const __nv_bfloat16* noise, int M, int H, float* h, float* hstat,
                          const float* w, float* hmax, const __nv_bfloat16* anchor, int block,
                          cudaStream_t st);
cudaError_t ctx_norm_launch(const float* raw, const float* part, int nparts, int rows, int H,
                            const float* w, float eps, __half* out, cudaStream_t st);
// hn: bf16 [M, H], or with drop_first the rows j >= 1 of every block of
// `block` rows, packed (row 0 of each block is not written)
cudaError_t final_norm_launch(const float* h, const float* hstat, int hparts, int M, int H,
                              const float* w, float eps, __nv_bfloat16* hn, void* out, bool out_f32,
                              cudaStream_t st, int block = 1, int drop_first = 0);
cudaError_t i8_to_f16_rows_launch(const int8_t* src, int rows, int K, __half* dst, int grp, int period,
                                   int off, cudaStream_t st);
// one bounded mbarrier wait that nothing completes: raises kDevMbarTimeout in *err
cudaError_t bounded_wait_probe_launch(uint32_t polls, int* err, cudaStream_t st);
cudaError_t i8_to_bf16_launch(const int8_t* src, size_t n, __nv_bfloat16* dst, cudaStream_t st);
cudaError_t i8_to_f16_launch(const int8_t* src, size_t n, __half* dst, cudaStream_t st);

// ---- fp32-accumulate path (f32_path.cu): fp32 weights and activations on the
// CUDA cores.  GEMM epilogues (after the ordered split-K sum):
//   kF32Store  : out = A . B^T
//   kF32Add    : out += A . B^T (the residual stream)
//   kF32Silu   : B holds the gate rows then the up rows; out = silu(g) * u
//   kF32Argmax : per-row (max, first index) over each 128-column tile into
//                best_val / best_idx [N tiles][M] (no split, no partials)
enum F32Mode : int { kF32Store = 0, kF32Add = 1, kF32Silu = 2, kF32Argmax = 3 };

struct F32GemmParams {
  int M, N, K;          // A [M, K], B [N, K] fp32 row-major; K % 64 == 0
  float* part;          // split-K partials [S][M][N]
  size_t part_floats;
  float* best_val;      // kF32Argmax
  int* best_idx;
  int* err;             // device error word for bounded waits
};

struct F32AttnParams {
  const float* q; int q_ld;               // block row m, head h at q + m * q_ld + h * 128
  const float* kc; const float* vc; int c_ld;   // context rows (packed), kv head hk at + hk * 128
  const float* kb; const float* vb; int b_ld;   // block rows
  const KvSeq* seq;                       // device records: ctx_start of each sequence (+ total)
  int nseq, block, nq, nkv;
  int chunk, splits;                      // keys per split (a multiple of 32), splits
  float scale;                            // head_dim^-0.5
  float *opart, *mpart, *lpart;           // [nseq][nq][splits][block] (x 128 for opart)
  float* out; int out_ld;                 // [M, NQ * 128]
};

int f32_gemm_splits(int M, int N, int K, int num_sms, size_t part_floats);
// the GEMM (+ the split reduction and epilogue into out[M, ldo], except kF32Argmax)
cudaError_t f32_gemm_launch(const float* A, const float* B, int mode, F32GemmParams p, float* out, int ldo,
                            int num_sms, cudaStream_t st);
// y = rms_norm(x) (if y); y2 = its rows j >= 1 of every block, packed (if y2)
cudaError_t f32_rmsnorm_launch(const float* x, int rows, int H, const float* w, float eps, float* y, float* y2,
                               int block, cudaStream_t st);
// per-head RMSNorm + neox RoPE in place: heads [0, nq) with wq, [nq, nq + nk) with
// wk (+ plane * 128), in `planes` column planes plane_cols apart; table row rope_row0 + row
cudaError_t f32_headnorm_launch(float* x, int rows, int ld, int nq, int nk, int planes, int plane_cols,
                                const float* wq, const float* wk, const float2* rope, int rope_row0, float eps,
                                int num_sms, cudaStream_t st);
void f32_attn_pick_split(int nseq, int nq, int kv_len_max, int num_sms, int max_splits, int* chunk, int* splits);
cudaError_t f32_attn_launch(const F32AttnParams& p, int num_sms, cudaStream_t st);
}  // namespace dfl
