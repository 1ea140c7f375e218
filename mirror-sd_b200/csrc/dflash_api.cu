// C ABI (include/dflash_b200.h): handle with device-resident weights and
// workspace, the stateless draft step, and the kernel-level entry points.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/dflash_b200.h"
#include "kernels.cuh"

using namespace dfl;

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define CK(call)                                                                        \
  do {                                                                                  \
    cudaError_t e_ = (call);                                                            \
    if (e_ != cudaSuccess) {                                                            \
      if (e_ == cudaErrorInvalidValue)                                                  \
        return fail(DFLASH_ERR_INVALID, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                    __FILE__, __LINE__);                                                \
      return fail(e_ == cudaErrorMemoryAllocation ? DFLASH_ERR_OOM : DFLASH_ERR_CUDA,   \
                  "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__);  \
    }                                                                                   \
  } while (0)

// device allocations owned by a handle, released together
struct Arena {
  std::vector<void*> ptrs;
  template <class T>
  cudaError_t alloc(T** p, size_t count) {
    void* q = nullptr;
    cudaError_t e = cudaMalloc(&q, count * sizeof(T) > 0 ? count * sizeof(T) : 16);
    if (e != cudaSuccess) return e;
    ptrs.push_back(q);
    *p = static_cast<T*>(q);
    return cudaSuccess;
  }
  void release() {
    for (void* p : ptrs) cudaFree(p);
    ptrs.clear();
  }
};

struct Layer {
  int8_t* w_qkv; float* s_qkv;   // tile-packed int8, channels [q heads | k heads | v heads]
  int8_t* w_o; float* s_o;
  int8_t* w_gu; float* s_gu;     // per 128-row tile: 64 gate rows then the matching 64 up rows
  int8_t* w_d; float* s_d;
  float *in_norm, *post_norm, *q_norm;
  // dense block path (handles whose max_batch * max_block exceeds kW8Rows):
  // exact f16 copies of the int8 weights, row-major [N, K]; gate|up
  // interleaved per 256 rows (128 gate rows, then the 128 matching up rows)
  __half *dw_qkv = nullptr, *dw_o = nullptr, *dw_gu = nullptr, *dw_d = nullptr;
  float* ds_gu = nullptr;
};

struct Handle {
  int device = 0;
  int num_sms = 148;
  int max_splits = 8;
  DFlashDims d{};
  Arena arena;
  std::mutex mu;
  // weights
  __nv_bfloat16* fc = nullptr;
  uint8_t* lm_tiles = nullptr;      // lm_head packed by lm_pack_launch (128-row swizzled tiles)
  float *hidden_norm = nullptr, *norm = nullptr, *inv_freq = nullptr;
  float* k_norm_all = nullptr;     // [L, 128]
  __half* w_kv_ctx = nullptr;       // [L*2*NKV*128, H] exact f16 of the int8 K|V weights
  float* s_kv_ctx = nullptr;       // [L*2*NKV*128]
  std::vector<Layer> layers;
  // workspace
  float2* rope = nullptr;
  float *h = nullptr, *hstat = nullptr;
  float* ctx_part = nullptr;        // per-256-column sums of squares of the fc rows [H/256, Cx]
  float* ctx_raw = nullptr;         // fc output [Cx, H] fp32
  __half* ctx_n = nullptr;          // hidden_norm(fc rows) in f16: the context K|V GEMM's A
  __half *K = nullptr, *V = nullptr, *Q = nullptr, *attn_out = nullptr, *act = nullptr;
  float* act_w8 = nullptr;          // W8A16 path: silu(g) * u rows in fp32 [min(Mx, 64), I]
  int8_t* xl = nullptr;             // projection input limbs [3][64][max(H, NQ*128, I)]
  float* xs = nullptr;              // their row scales [64]
  float* hmax = nullptr;            // [H/128, Mx] partial max |h * next norm weight|
  float* amax = nullptr;            // [max(NQ, 2I/128), Mx] partial max |attention out| / |act|
  float *opart = nullptr, *mpart = nullptr, *lpart = nullptr;
  size_t attn_part_rows = 0;
  __nv_bfloat16* hn = nullptr;
  float* lm_val = nullptr;
  int* lm_idx = nullptr;
  int* dev_err = nullptr;
  float* w8_part = nullptr;          // split-K partials of the W8A16 projections
  size_t w8_part_floats = 0;
  int* w8_cnt = nullptr;             // per-tile arrival counters (zero between launches)
  __nv_bfloat16* anchor = nullptr;   // [max_batch, H] soft anchor rows
  float* sa_cand_v = nullptr;        // [max_batch, kSaMaxCtas, kSaMaxK] soft anchor candidates
  int* sa_cand_i = nullptr;
  int* sa_cnt = nullptr;             // [max_batch] arrival counters (zero between launches)
  KvSeq* kv_seq = nullptr;           // [max_batch + 1] per-sequence records of the current forward
  float* tc_part = nullptr;          // tcgen05 GEMM tail-split partials [tc_cap][128 * 256]
  int tc_cap = 0;
  int* tc_cnt = nullptr;             // their arrival counters [num_sms] (zero between launches)
  bool dense = false;                // the dense block path is available (max rows > kW8Rows)
  size_t stateless_rows = 0;         // K/V rows per layer and kv head of the stateless store
  __half* xa = nullptr;              // dense path: normalised projection input [Mx, H] f16
  int last_launches = 0;
  // fp32-accumulate mode (dflash_create_f32): fp32 weights, activations and sums
  bool f32 = false;
  struct LayerF32 {
    float* w_qkv = nullptr;          // [(NQ + 2 NKV) * 128, H]: q rows, k rows, v rows
    float* w_o = nullptr;            // [H, NQ * 128]
    float* w_gu = nullptr;           // [2 I, H]: gate rows, then up rows
    float* w_d = nullptr;            // [H, I]
  };
  std::vector<LayerF32> flayers;
  float* f_fc = nullptr;             // [H, F * H]
  float* f_lm = nullptr;             // [V, H]
  float* f_wkv = nullptr;            // [L][2 * NKV * 128][H]: every layer's k rows then v rows
  float *f_ctx = nullptr, *f_ctxn = nullptr;   // fc output and its hidden_norm [Cx, H]
  float* f_kvc = nullptr;            // context K | V of the step's layers [Cx, nl * 2 * NKV * 128]
  float *f_h = nullptr, *f_xn = nullptr;        // residual stream, normed rows [Mx, H]
  float* f_qkv = nullptr;            // block q | k | v [Mx, (NQ + 2 NKV) * 128]
  float* f_attn = nullptr;           // [Mx, NQ * 128]
  float* f_act = nullptr;            // [Mx, I]
  float* f_hn = nullptr;             // final-normed rows j >= 1 of every block [Mx, H]
  float* f_part = nullptr;           // GEMM split partials
  size_t f_part_floats = 0;
  float *f_opart = nullptr, *f_mpart = nullptr, *f_lpart = nullptr;   // attention split partials
  size_t f_attn_rows = 0;
};

// Draft KV cache (dflash.py:139-212).  Per layer and sequence the host keeps
// the logical state; the device holds the rows in the KvMap ring layout of
// kernels.cuh ([layer][sequence][kv head][slot][128] f16).
struct SeqState {
  int offset = 0;  // positions processed (RoPE offset), dflash.py:172
  int hl = 0;      // rows in the sink slots
  int rs = 0;      // ring start
  int rl = 0;      // rows in the ring
  bool operator==(const SeqState& o) const {
    return offset == o.offset && hl == o.hl && rs == o.rs && rl == o.rl;
  }
};

struct Cache {
  const Handle* owner = nullptr;    // compared, never dereferenced: the cache may outlive it
  int device = 0, nkv = 0;
  std::mutex mu;                    // host state; dflash_forward takes it after the handle's
  int layers = 0, max_batch = 0;
  int sink_size = 0, window_size = 0;
  bool evict = false;               // sink_size > 0 && window_size > 0 (dflash.py:180-181)
  int sink = 0, ring = 0, slots = 0;
  __half *K = nullptr, *V = nullptr;
  size_t layer_stride = 0;          // halves
  std::vector<SeqState> st;         // [layers][max_batch]
  SeqState& at(int l, int s) { return st[(size_t)l * max_batch + s]; }
};

// block rows one forward may carry; above kW8Rows the projections and the
// lm_head run as dense tcgen05 GEMMs over exact f16 copies of the weights
constexpr int kW8Rows = 64;
constexpr int kMaxBlockRows = 16384;

// DFlashKVCache.trim (dflash.py:200-208) on one sequence's state
void trim_state(SeqState& q, int n) {
  if (n <= 0) return;
  const int len = std::max(q.hl + q.rl - n, 0);  // dflash.py:204
  if (len >= q.hl) {
    q.rl = len - q.hl;
  } else {
    q.rl = 0;
    q.hl = len;
  }
  q.offset -= n;                                 // dflash.py:207
}

// context rows one forward may carry (all sequences)
int ctx_rows_capacity(const DFlashDims& d) {
  return d.max_ctx_rows > 0 ? d.max_ctx_rows : d.max_batch * d.max_ctx;
}

int check_dims(const DFlashDims* d) {
  if (!d) return fail(DFLASH_ERR_INVALID, "dims is NULL");
  if (d->head_dim != 128) return fail(DFLASH_ERR_INVALID, "head_dim must be 128 (got %d)", d->head_dim);
  if (d->hidden_size <= 0 || d->hidden_size % 256)
    return fail(DFLASH_ERR_INVALID, "hidden_size must be a positive multiple of 256 (got %d)", d->hidden_size);
  if (d->intermediate_size <= 0 || d->intermediate_size % 128)
    return fail(DFLASH_ERR_INVALID, "intermediate_size must be a multiple of 128 (got %d)", d->intermediate_size);
  if (d->num_attention_heads <= 0 || d->num_key_value_heads <= 0 ||
      d->num_attention_heads % d->num_key_value_heads)
    return fail(DFLASH_ERR_INVALID, "num_attention_heads must be a multiple of num_key_value_heads");
  if ((d->num_attention_heads + 2 * d->num_key_value_heads) % 2)
    return fail(DFLASH_ERR_INVALID, "num_attention_heads + 2*num_key_value_heads must be even");
  if (d->num_hidden_layers < 1 || d->vocab_size < 1 || d->num_target_features < 1)
    return fail(DFLASH_ERR_INVALID, "layers, vocab and target features must be positive");
  if (d->max_batch < 1 || d->max_block < 2 || d->max_block > 1024 || d->max_ctx < 0 ||
      (long long)d->max_batch * d->max_block > kMaxBlockRows)
    return fail(DFLASH_ERR_INVALID, "capacities: max_batch*max_block must be in [2, %d], max_ctx >= 0",
                kMaxBlockRows);
  if (d->max_ctx_rows < 0 || (d->max_ctx_rows == 0 && (long long)d->max_batch * d->max_ctx > (1LL << 30)) ||
      (d->max_ctx_rows > 0 && d->max_ctx_rows < d->max_ctx))
    return fail(DFLASH_ERR_INVALID, "max_ctx_rows %d: must be 0 (max_batch * max_ctx <= 2^30) or >= max_ctx",
                d->max_ctx_rows);
  const int G = d->num_attention_heads / d->num_key_value_heads;
  if (G * d->max_block > 192)
    return fail(DFLASH_ERR_INVALID, "query rows per kv head (heads/kv_heads * block) must be <= 192");
  return DFLASH_OK;
}

size_t attn_rows_capacity(int max_batch, int nkv, int R, int kv_len_max, int num_sms) {
  size_t best = 0;
  for (int b = 1; b <= max_batch; ++b) {
    (void)kv_len_max;
    // attn_max_splits bounds the split count at every kv length
    const size_t rows = (size_t)b * nkv * attn_max_splits(b, nkv, num_sms, R) * R;
    if (rows > best) best = rows;
  }
  return best;
}

constexpr int kF32MaxAttnSplits = 16;

// attention split partial rows an fp32 handle needs: only steps with more
// than one split use them
size_t f32_attn_rows_capacity(int max_batch, int nq, int block, int num_sms) {
  size_t best = 0;
  for (int b = 1; b <= max_batch; ++b) {
    int chunk, splits;
    f32_attn_pick_split(b, nq, 1 << 28, num_sms, kF32MaxAttnSplits, &chunk, &splits);
    if (splits > 1) best = std::max(best, (size_t)b * nq * splits * block);
  }
  return best;
}

// The fp32-accumulate draft step (DFlashDraftModel.__call__, dflash.py:384-403,
// then lm_head + greedy argmax + acceptance, generate.py:604-606, :722-728),
// stateless: sequence s attends to its C_s context rows and its block rows.
int forward_f32(Handle* hd, const DFlashForwardArgs* a, std::vector<KvSeq>& sq, cudaStream_t st) {
  const DFlashDims& d = hd->d;
  const int H = d.hidden_size, I = d.intermediate_size, NQ = d.num_attention_heads,
            NKV = d.num_key_value_heads, F = d.num_target_features;
  const int b = a->batch, B = a->block, nl = a->num_layers;
  const int M = b * B;
  const int Ctot = sq[b].ctx_start;
  if (a->cache || a->anchor_logits || a->target_layers)
    return fail(DFLASH_ERR_INVALID, "cache, anchor_logits and target_layers are not available on an fp32 handle");
  if (M > kMaxBlockRows) return fail(DFLASH_ERR_INVALID, "%d block rows above %d", M, kMaxBlockRows);
  if ((reinterpret_cast<uintptr_t>(a->noise) | reinterpret_cast<uintptr_t>(a->target_hidden) |
       reinterpret_cast<uintptr_t>(a->out_hidden)) & 15)
    return fail(DFLASH_ERR_INVALID, "noise, target_hidden and out_hidden must be 16-byte aligned");
  KvMap m{};
  m.nseq = b;
  m.seq = hd->kv_seq;
  m.sink = 0;
  int kvmax = 0;
  for (int s = 0; s < b; ++s) {
    const int off = a->rope_offsets ? a->rope_offsets[s] : a->rope_offset;
    if (off < 0) return fail(DFLASH_ERR_INVALID, "rope offsets must be >= 0");
    sq[s].n0 = 0; sq[s].rs_pre = 0; sq[s].rs_post = 0;
    sq[s].n_att = sq[s + 1].ctx_start - sq[s].ctx_start + B;
    sq[s].pos0 = off;
    sq[s].cseq = s;
    kvmax = std::max(kvmax, sq[s].n_att);
  }
  m.ring = m.slots = kvmax;
  std::lock_guard<std::mutex> lock(hd->mu);
  CK(cudaSetDevice(hd->device));
  const bool timing = a->phase_events && a->n_phase_events >= DFLASH_PHASES;
  auto mark = [&](int k) -> cudaError_t {
    return timing ? cudaEventRecord(static_cast<cudaEvent_t>(a->phase_events[k]), st) : cudaSuccess;
  };
  const int sms = hd->num_sms;
  const float eps = d.rms_norm_eps;
  int launches = 0;
  F32GemmParams gp{};
  gp.part = hd->f_part; gp.part_floats = hd->f_part_floats; gp.err = hd->dev_err;
  auto gemm = [&](const float* A, int Mr, const float* Bw, int N, int K, int mode, float* out, int ldo) {
    F32GemmParams p = gp;
    p.M = Mr; p.N = N; p.K = K;
    launches += 2;
    return f32_gemm_launch(A, Bw, mode, p, out, ldo, sms, st);
  };
  CK(mark(0));
  CK(rope_table_map_launch(m, sq.data(), B, hd->inv_freq, hd->rope, st));
  if (b + 1 > kKvChunk) launches += (b + kKvChunk) / kKvChunk;
  CK(cudaMemcpyAsync(hd->f_h, a->noise, (size_t)M * H * sizeof(float), cudaMemcpyDeviceToDevice, st));
  launches += 1;
  CK(mark(1));
  const int nkv2 = 2 * NKV * 128;
  const int ld_kvc = nl * nkv2;
  if (Ctot > 0) {
    CK(gemm(reinterpret_cast<const float*>(a->target_hidden), Ctot, hd->f_fc, H, F * H, kF32Store, hd->f_ctx, H));
    CK(mark(2));
    CK(f32_rmsnorm_launch(hd->f_ctx, Ctot, H, hd->hidden_norm, eps, hd->f_ctxn, nullptr, 1, st));
    CK(mark(3));
    CK(gemm(hd->f_ctxn, Ctot, hd->f_wkv, ld_kvc, H, kF32Store, hd->f_kvc, ld_kvc));
    CK(f32_headnorm_launch(hd->f_kvc, Ctot, ld_kvc, 0, NKV, nl, nkv2, nullptr, hd->k_norm_all, hd->rope, 0, eps,
                           sms, st));
    launches += 2;
  } else {
    CK(mark(2));
    CK(mark(3));
  }
  CK(mark(4));
  const int nqkv = (NQ + 2 * NKV) * 128;
  F32AttnParams ap{};
  ap.q = hd->f_qkv; ap.q_ld = nqkv;
  ap.c_ld = ld_kvc;
  ap.kb = hd->f_qkv + NQ * 128; ap.vb = hd->f_qkv + (NQ + NKV) * 128; ap.b_ld = nqkv;
  ap.seq = hd->kv_seq; ap.nseq = b; ap.block = B; ap.nq = NQ; ap.nkv = NKV;
  f32_attn_pick_split(b, NQ, kvmax, sms, kF32MaxAttnSplits, &ap.chunk, &ap.splits);
  if (ap.splits > 1 && (size_t)b * NQ * ap.splits * B > hd->f_attn_rows)
    return fail(DFLASH_ERR_INVALID, "attention workspace too small");
  ap.scale = (float)(1.0 / std::sqrt(128.0));
  ap.opart = hd->f_opart; ap.mpart = hd->f_mpart; ap.lpart = hd->f_lpart;
  ap.out = hd->f_attn; ap.out_ld = NQ * 128;
  for (int l = 0; l < nl; ++l) {
    const Layer& ly = hd->layers[l];
    const Handle::LayerF32& fl = hd->flayers[l];
    CK(f32_rmsnorm_launch(hd->f_h, M, H, ly.in_norm, eps, hd->f_xn, nullptr, 1, st));
    CK(gemm(hd->f_xn, M, fl.w_qkv, nqkv, H, kF32Store, hd->f_qkv, nqkv));
    CK(f32_headnorm_launch(hd->f_qkv, M, nqkv, NQ, NKV, 1, 0, ly.q_norm, hd->k_norm_all + l * 128, hd->rope, Ctot,
                           eps, sms, st));
    ap.kc = hd->f_kvc + (size_t)l * nkv2;
    ap.vc = ap.kc + NKV * 128;
    CK(f32_attn_launch(ap, sms, st));
    CK(gemm(hd->f_attn, M, fl.w_o, H, NQ * 128, kF32Add, hd->f_h, H));
    CK(f32_rmsnorm_launch(hd->f_h, M, H, ly.post_norm, eps, hd->f_xn, nullptr, 1, st));
    CK(gemm(hd->f_xn, M, fl.w_gu, 2 * I, H, kF32Silu, hd->f_act, I));
    CK(gemm(hd->f_act, M, fl.w_d, H, I, kF32Add, hd->f_h, H));
    launches += 4 + (ap.splits > 1);
  }
  CK(mark(5));
  const bool lm = a->out_tokens || a->target_tokens;
  CK(f32_rmsnorm_launch(hd->f_h, M, H, hd->norm, eps, static_cast<float*>(a->out_hidden), lm ? hd->f_hn : nullptr,
                        B, st));
  launches += 1;
  CK(mark(6));
  if (lm) {
    F32GemmParams p = gp;
    p.M = b * (B - 1); p.N = d.vocab_size; p.K = H;
    p.best_val = hd->lm_val; p.best_idx = hd->lm_idx;
    CK(f32_gemm_launch(hd->f_hn, hd->f_lm, kF32Argmax, p, nullptr, 0, sms, st));
    const int parts = (d.vocab_size + 127) / 128;
    CK(argmax_accept_launch(hd->lm_val, hd->lm_idx, parts, b * (B - 1), B, b, a->out_tokens, a->target_tokens,
                            a->acc_len, a->correction, st, 1));
    launches += 2;
  }
  CK(mark(7));
  hd->last_launches = launches;
  return DFLASH_OK;
}

}  // namespace

extern "C" {

int dflash_version(void) { return 1; }

int dflash_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return (int)g_err.size();
  snprintf(buf, len, "%s", g_err.c_str());
  return (int)g_err.size();
}

int dflash_create(const DFlashDims* dims, const DFlashWeightsView* w, int device, void** out) {
  if (int r = check_dims(dims)) return r;
  if (!w || !out || !w->fc || !w->hidden_norm || !w->norm || !w->lm_head || !w->layers)
    return fail(DFLASH_ERR_INVALID, "weights view has NULL members");
  const DFlashDims d = *dims;
  const int H = d.hidden_size, I = d.intermediate_size, NQ = d.num_attention_heads,
            NKV = d.num_key_value_heads, L = d.num_hidden_layers, F = d.num_target_features;
  for (int l = 0; l < L; ++l) {
    const DFlashLayerWeights& lw = w->layers[l];
    if (!lw.wq || !lw.sq || !lw.wk || !lw.sk || !lw.wv || !lw.sv || !lw.wo || !lw.so || !lw.wg ||
        !lw.sg || !lw.wu || !lw.su || !lw.wd || !lw.sd || !lw.input_layernorm ||
        !lw.post_attention_layernorm || !lw.q_norm || !lw.k_norm)
      return fail(DFLASH_ERR_INVALID, "layer %d has NULL weight pointers", l);
  }
  CK(cudaSetDevice(device));
  Handle* hd = new Handle();
  hd->device = device;
  hd->d = d;
  int rc = DFLASH_OK;
  auto cleanup = [&]() {
    cudaDeviceSynchronize();
    hd->arena.release();
    delete hd;
  };
#define CKC(call)                         \
  do {                                    \
    cudaError_t e_ = (call);              \
    if (e_ != cudaSuccess) {              \
      rc = fail(e_ == cudaErrorMemoryAllocation ? DFLASH_ERR_OOM : DFLASH_ERR_CUDA, "%s: %s", #call, \
                cudaGetErrorString(e_));  \
      cleanup();                          \
      return rc;                          \
    }                                     \
  } while (0)
  CKC(cudaDeviceGetAttribute(&hd->num_sms, cudaDevAttrMultiProcessorCount, device));
  Arena& A = hd->arena;
  cudaStream_t st = 0;
  // ---- weights
  const size_t fc_elems = (size_t)H * F * H;
  CKC(A.alloc(&hd->fc, fc_elems));
  CKC(cudaMemcpyAsync(hd->fc, w->fc, fc_elems * 2, cudaMemcpyDeviceToDevice, st));
  CKC(A.alloc(&hd->lm_tiles, lm_pack_bytes(d.vocab_size, H)));
  CKC(lm_pack_launch(reinterpret_cast<const __nv_bfloat16*>(w->lm_head), d.vocab_size, H, hd->lm_tiles, st));
  CKC(A.alloc(&hd->hidden_norm, H));
  CKC(A.alloc(&hd->norm, H));
  CKC(cudaMemcpyAsync(hd->hidden_norm, w->hidden_norm, H * 4, cudaMemcpyDeviceToDevice, st));
  CKC(cudaMemcpyAsync(hd->norm, w->norm, H * 4, cudaMemcpyDeviceToDevice, st));
  {
    std::vector<float> inv(64);
    for (int i = 0; i < 64; ++i) inv[i] = (float)std::pow((double)d.rope_theta, -2.0 * i / 128.0);
    CKC(A.alloc(&hd->inv_freq, 64));
    CKC(cudaMemcpy(hd->inv_freq, inv.data(), 64 * 4, cudaMemcpyHostToDevice));
  }
  const int nqkv = (NQ + 2 * NKV) * 128;
  const int nkvc = 2 * NKV * 128;
  CKC(A.alloc(&hd->k_norm_all, (size_t)L * 128));
  CKC(A.alloc(&hd->w_kv_ctx, (size_t)L * nkvc * H));
  CKC(A.alloc(&hd->s_kv_ctx, (size_t)L * nkvc));
  const int big = 1 << 30;
  for (int l = 0; l < L; ++l) {
    const DFlashLayerWeights& lw = w->layers[l];
    Layer ly{};
    CKC(A.alloc(&ly.w_qkv, (size_t)nqkv * H));
    CKC(A.alloc(&ly.s_qkv, nqkv));
    CKC(w8_tilepack_launch(lw.wq, NQ * 128, H, ly.w_qkv, big, 0, 0, st));
    CKC(w8_tilepack_launch(lw.wk, NKV * 128, H, ly.w_qkv, big, 0, NQ * 128, st));
    CKC(w8_tilepack_launch(lw.wv, NKV * 128, H, ly.w_qkv, big, 0, (NQ + NKV) * 128, st));
    CKC(w8_scale_launch((const __half*)lw.sq, NQ * 128, ly.s_qkv, big, 0, 0, st));
    CKC(w8_scale_launch((const __half*)lw.sk, NKV * 128, ly.s_qkv, big, 0, NQ * 128, st));
    CKC(w8_scale_launch((const __half*)lw.sv, NKV * 128, ly.s_qkv, big, 0, (NQ + NKV) * 128, st));
    CKC(A.alloc(&ly.w_o, (size_t)H * NQ * 128));
    CKC(A.alloc(&ly.s_o, H));
    CKC(w8_tilepack_launch(lw.wo, H, NQ * 128, ly.w_o, big, 0, 0, st));
    CKC(w8_scale_launch((const __half*)lw.so, H, ly.s_o, big, 0, 0, st));
    // gate/up interleaved per 128-channel tile: 64 gate channels then the 64 matching up channels
    CKC(A.alloc(&ly.w_gu, (size_t)2 * I * H));
    CKC(A.alloc(&ly.s_gu, 2 * I));
    CKC(w8_tilepack_launch(lw.wg, I, H, ly.w_gu, 64, 128, 0, st));
    CKC(w8_tilepack_launch(lw.wu, I, H, ly.w_gu, 64, 128, 64, st));
    CKC(w8_scale_launch((const __half*)lw.sg, I, ly.s_gu, 64, 128, 0, st));
    CKC(w8_scale_launch((const __half*)lw.su, I, ly.s_gu, 64, 128, 64, st));
    CKC(A.alloc(&ly.w_d, (size_t)H * I));
    CKC(A.alloc(&ly.s_d, H));
    CKC(w8_tilepack_launch(lw.wd, H, I, ly.w_d, big, 0, 0, st));
    CKC(w8_scale_launch((const __half*)lw.sd, H, ly.s_d, big, 0, 0, st));
    CKC(A.alloc(&ly.in_norm, H));
    CKC(A.alloc(&ly.post_norm, H));
    CKC(A.alloc(&ly.q_norm, 128));
    CKC(cudaMemcpyAsync(ly.in_norm, lw.input_layernorm, H * 4, cudaMemcpyDeviceToDevice, st));
    CKC(cudaMemcpyAsync(ly.post_norm, lw.post_attention_layernorm, H * 4, cudaMemcpyDeviceToDevice, st));
    CKC(cudaMemcpyAsync(ly.q_norm, lw.q_norm, 128 * 4, cudaMemcpyDeviceToDevice, st));
    CKC(cudaMemcpyAsync(hd->k_norm_all + l * 128, lw.k_norm, 128 * 4, cudaMemcpyDeviceToDevice, st));
    // context K|V operand: exact f16 of the int8 values, scales applied in the epilogue
    __half* kv = hd->w_kv_ctx + (size_t)l * nkvc * H;
    CKC(i8_to_f16_launch(lw.wk, (size_t)NKV * 128 * H, kv, st));
    CKC(i8_to_f16_launch(lw.wv, (size_t)NKV * 128 * H, kv + (size_t)NKV * 128 * H, st));
    CKC(w8_scale_launch((const __half*)lw.sk, NKV * 128, hd->s_kv_ctx + (size_t)l * nkvc, big, 0, 0, st));
    CKC(w8_scale_launch((const __half*)lw.sv, NKV * 128, hd->s_kv_ctx + (size_t)l * nkvc, big, 0, NKV * 128, st));
    if ((long long)d.max_batch * d.max_block > kW8Rows) {
      CKC(A.alloc(&ly.dw_qkv, (size_t)nqkv * H));
      CKC(i8_to_f16_launch(lw.wq, (size_t)NQ * 128 * H, ly.dw_qkv, st));
      CKC(i8_to_f16_launch(lw.wk, (size_t)NKV * 128 * H, ly.dw_qkv + (size_t)NQ * 128 * H, st));
      CKC(i8_to_f16_launch(lw.wv, (size_t)NKV * 128 * H, ly.dw_qkv + (size_t)(NQ + NKV) * 128 * H, st));
      CKC(A.alloc(&ly.dw_o, (size_t)H * NQ * 128));
      CKC(i8_to_f16_launch(lw.wo, (size_t)H * NQ * 128, ly.dw_o, st));
      CKC(A.alloc(&ly.dw_gu, (size_t)2 * I * H));
      CKC(i8_to_f16_rows_launch(lw.wg, I, H, ly.dw_gu, 128, 256, 0, st));
      CKC(i8_to_f16_rows_launch(lw.wu, I, H, ly.dw_gu, 128, 256, 128, st));
      CKC(A.alloc(&ly.ds_gu, 2 * I));
      CKC(w8_scale_launch((const __half*)lw.sg, I, ly.ds_gu, 128, 256, 0, st));
      CKC(w8_scale_launch((const __half*)lw.su, I, ly.ds_gu, 128, 256, 128, st));
      CKC(A.alloc(&ly.dw_d, (size_t)H * I));
      CKC(i8_to_f16_launch(lw.wd, (size_t)H * I, ly.dw_d, st));
    }
    hd->layers.push_back(ly);
  }
  // ---- workspace
  const int Mx = d.max_batch * d.max_block;
  const int Cx = ctx_rows_capacity(d);
  const int G = NQ / NKV;
  hd->stateless_rows = (size_t)Cx + Mx;
  CKC(A.alloc(&hd->rope, (size_t)(Cx + Mx) * 64));
  CKC(A.alloc(&hd->h, (size_t)Mx * H));
  CKC(A.alloc(&hd->hstat, (size_t)(H / 128) * Mx));
  if (Cx > 0) {
    CKC(A.alloc(&hd->ctx_part, (size_t)(H / 256) * Cx));
    CKC(A.alloc(&hd->ctx_raw, (size_t)Cx * H));
    CKC(A.alloc(&hd->ctx_n, (size_t)Cx * H));
  }
  const size_t kv_elems = (size_t)L * NKV * hd->stateless_rows * 128;
  CKC(A.alloc(&hd->K, kv_elems));
  CKC(A.alloc(&hd->V, kv_elems));
  CKC(A.alloc(&hd->Q, (size_t)Mx * NQ * 128));
  CKC(A.alloc(&hd->attn_out, (size_t)Mx * NQ * 128));
  CKC(A.alloc(&hd->act, (size_t)Mx * I));
  CKC(A.alloc(&hd->act_w8, (size_t)std::min(Mx, kW8Rows) * I));
  CKC(A.alloc(&hd->xl, (size_t)3 * 64 * std::max(std::max(H, NQ * 128), I)));
  CKC(A.alloc(&hd->xs, 64));
  CKC(A.alloc(&hd->hmax, (size_t)(H / 128) * Mx));
  CKC(A.alloc(&hd->amax, (size_t)std::max(NQ, 2 * I / 128) * Mx));
  // the split count never exceeds what the longest rows give, and a cache can
  // make rows longer than max_ctx + max_block: size for any length
  hd->attn_part_rows = attn_rows_capacity(d.max_batch, NKV, G * d.max_block, 1 << 28, hd->num_sms);
  CKC(A.alloc(&hd->opart, hd->attn_part_rows * 128));
  CKC(A.alloc(&hd->mpart, hd->attn_part_rows));
  CKC(A.alloc(&hd->lpart, hd->attn_part_rows));
  CKC(A.alloc(&hd->hn, (size_t)Mx * H));
  hd->dense = Mx > kW8Rows;
  // lm_head argmax partials: one per CTA (W8 path) or per 256-entry vocabulary block (dense path)
  const size_t lm_parts = std::max<size_t>(hd->num_sms, (d.vocab_size + 255) / 256);
  CKC(A.alloc(&hd->lm_val, lm_parts * Mx));
  CKC(A.alloc(&hd->lm_idx, lm_parts * Mx));
  if (hd->dense) CKC(A.alloc(&hd->xa, (size_t)Mx * H));
  {
    const int shapes[4][2] = {{(NQ + 2 * NKV) * 128, H}, {H, NQ * 128}, {2 * I, H}, {H, I}};
    int max_tiles = 0;
    for (auto& sh : shapes) {
      const size_t f = w8tc_part_floats(sh[0], sh[1], std::min(Mx, kW8Rows), hd->num_sms);
      if (f > hd->w8_part_floats) hd->w8_part_floats = f;
      if (sh[0] / 128 > max_tiles) max_tiles = sh[0] / 128;
    }
    CKC(A.alloc(&hd->w8_part, hd->w8_part_floats));
    CKC(A.alloc(&hd->w8_cnt, (size_t)max_tiles));
    CKC(cudaMemset(hd->w8_cnt, 0, (size_t)max_tiles * sizeof(int)));
  }
  CKC(A.alloc(&hd->dev_err, 1));
  CKC(cudaMemset(hd->dev_err, 0, sizeof(int)));
  {
    const size_t nc = (size_t)d.max_batch * kSaMaxCtas * kSaMaxK;
    CKC(A.alloc(&hd->anchor, (size_t)d.max_batch * H));
    CKC(A.alloc(&hd->sa_cand_v, nc));
    CKC(A.alloc(&hd->sa_cand_i, nc));
    CKC(A.alloc(&hd->sa_cnt, (size_t)d.max_batch));
    CKC(A.alloc(&hd->kv_seq, (size_t)d.max_batch + 1));
    hd->tc_cap = 4 * hd->num_sms;   // up to ~4 tail parts per CTA
    CKC(A.alloc(&hd->tc_part, (size_t)hd->tc_cap * 128 * 256));
    CKC(A.alloc(&hd->tc_cnt, (size_t)hd->num_sms));
    CKC(cudaMemset(hd->tc_cnt, 0, (size_t)hd->num_sms * sizeof(int)));
    CKC(cudaMemset(hd->sa_cnt, 0, (size_t)d.max_batch * sizeof(int)));
  }
  CKC(cudaDeviceSynchronize());
#undef CKC
  *out = hd;
  return DFLASH_OK;
}

int dflash_create_f32(const DFlashDims* dims, const DFlashWeightsViewF32* w, int device, void** out) {
  if (int r = check_dims(dims)) return r;
  if (!w || !out || !w->fc || !w->hidden_norm || !w->norm || !w->lm_head || !w->layers)
    return fail(DFLASH_ERR_INVALID, "weights view has NULL members");
  const DFlashDims d = *dims;
  const int H = d.hidden_size, I = d.intermediate_size, NQ = d.num_attention_heads,
            NKV = d.num_key_value_heads, L = d.num_hidden_layers, F = d.num_target_features, V = d.vocab_size;
  for (int l = 0; l < L; ++l) {
    const DFlashLayerWeightsF32& lw = w->layers[l];
    if (!lw.wq || !lw.wk || !lw.wv || !lw.wo || !lw.wg || !lw.wu || !lw.wd || !lw.input_layernorm ||
        !lw.post_attention_layernorm || !lw.q_norm || !lw.k_norm)
      return fail(DFLASH_ERR_INVALID, "layer %d has NULL weight pointers", l);
  }
  CK(cudaSetDevice(device));
  Handle* hd = new Handle();
  hd->device = device;
  hd->d = d;
  hd->f32 = true;
  int rc = DFLASH_OK;
  auto cleanup = [&]() {
    cudaDeviceSynchronize();
    hd->arena.release();
    delete hd;
  };
#define CKC(call)                                                                                    \
  do {                                                                                               \
    cudaError_t e_ = (call);                                                                         \
    if (e_ != cudaSuccess) {                                                                         \
      rc = fail(e_ == cudaErrorMemoryAllocation ? DFLASH_ERR_OOM : DFLASH_ERR_CUDA, "%s: %s", #call, \
                cudaGetErrorString(e_));                                                             \
      cleanup();                                                                                     \
      return rc;                                                                                     \
    }                                                                                                \
  } while (0)
  CKC(cudaDeviceGetAttribute(&hd->num_sms, cudaDevAttrMultiProcessorCount, device));
  Arena& A = hd->arena;
  cudaStream_t st = 0;
  auto copy = [&](float* dst, const float* src, size_t n) {
    return cudaMemcpyAsync(dst, src, n * sizeof(float), cudaMemcpyDeviceToDevice, st);
  };
  const size_t nqkv = (size_t)(NQ + 2 * NKV) * 128, nkv1 = (size_t)NKV * 128;
  CKC(A.alloc(&hd->f_fc, (size_t)H * F * H));
  CKC(copy(hd->f_fc, w->fc, (size_t)H * F * H));
  CKC(A.alloc(&hd->f_lm, (size_t)V * H));
  CKC(copy(hd->f_lm, w->lm_head, (size_t)V * H));
  CKC(A.alloc(&hd->hidden_norm, H));
  CKC(A.alloc(&hd->norm, H));
  CKC(copy(hd->hidden_norm, w->hidden_norm, H));
  CKC(copy(hd->norm, w->norm, H));
  {
    std::vector<float> inv(64);
    for (int i = 0; i < 64; ++i) inv[i] = (float)std::pow((double)d.rope_theta, -2.0 * i / 128.0);
    CKC(A.alloc(&hd->inv_freq, 64));
    CKC(cudaMemcpy(hd->inv_freq, inv.data(), 64 * 4, cudaMemcpyHostToDevice));
  }
  CKC(A.alloc(&hd->k_norm_all, (size_t)L * 128));
  CKC(A.alloc(&hd->f_wkv, (size_t)L * 2 * nkv1 * H));
  for (int l = 0; l < L; ++l) {
    const DFlashLayerWeightsF32& lw = w->layers[l];
    Handle::LayerF32 fl;
    CKC(A.alloc(&fl.w_qkv, nqkv * H));
    CKC(copy(fl.w_qkv, lw.wq, (size_t)NQ * 128 * H));
    CKC(copy(fl.w_qkv + (size_t)NQ * 128 * H, lw.wk, nkv1 * H));
    CKC(copy(fl.w_qkv + (size_t)(NQ + NKV) * 128 * H, lw.wv, nkv1 * H));
    CKC(A.alloc(&fl.w_o, (size_t)H * NQ * 128));
    CKC(copy(fl.w_o, lw.wo, (size_t)H * NQ * 128));
    CKC(A.alloc(&fl.w_gu, (size_t)2 * I * H));
    CKC(copy(fl.w_gu, lw.wg, (size_t)I * H));
    CKC(copy(fl.w_gu + (size_t)I * H, lw.wu, (size_t)I * H));
    CKC(A.alloc(&fl.w_d, (size_t)H * I));
    CKC(copy(fl.w_d, lw.wd, (size_t)H * I));
    float* kv = hd->f_wkv + (size_t)l * 2 * nkv1 * H;
    CKC(copy(kv, lw.wk, nkv1 * H));
    CKC(copy(kv + nkv1 * H, lw.wv, nkv1 * H));
    Layer ly{};
    CKC(A.alloc(&ly.in_norm, H));
    CKC(A.alloc(&ly.post_norm, H));
    CKC(A.alloc(&ly.q_norm, 128));
    CKC(copy(ly.in_norm, lw.input_layernorm, H));
    CKC(copy(ly.post_norm, lw.post_attention_layernorm, H));
    CKC(copy(ly.q_norm, lw.q_norm, 128));
    CKC(copy(hd->k_norm_all + l * 128, lw.k_norm, 128));
    hd->layers.push_back(ly);
    hd->flayers.push_back(fl);
  }
  // ---- workspace
  const int Mx = d.max_batch * d.max_block;
  const int Cx = ctx_rows_capacity(d);
  CKC(A.alloc(&hd->rope, (size_t)(Cx + Mx) * 64));
  if (Cx > 0) {
    CKC(A.alloc(&hd->f_ctx, (size_t)Cx * H));
    CKC(A.alloc(&hd->f_ctxn, (size_t)Cx * H));
    CKC(A.alloc(&hd->f_kvc, (size_t)Cx * L * 2 * nkv1));
  }
  CKC(A.alloc(&hd->f_h, (size_t)Mx * H));
  CKC(A.alloc(&hd->f_xn, (size_t)Mx * H));
  CKC(A.alloc(&hd->f_qkv, (size_t)Mx * nqkv));
  CKC(A.alloc(&hd->f_attn, (size_t)Mx * NQ * 128));
  CKC(A.alloc(&hd->f_act, (size_t)Mx * I));
  CKC(A.alloc(&hd->f_hn, (size_t)Mx * H));
  {
    // split partials: every GEMM of a step fits unsplit, and small ones may split
    size_t need = std::max({(size_t)Cx * H, (size_t)Cx * L * 2 * nkv1, (size_t)Mx * nqkv, (size_t)Mx * 2 * I,
                            (size_t)Mx * H});
    hd->f_part_floats = std::max(need, (size_t)8 << 20);
    CKC(A.alloc(&hd->f_part, hd->f_part_floats));
  }
  hd->f_attn_rows = f32_attn_rows_capacity(d.max_batch, NQ, d.max_block, hd->num_sms);
  if (hd->f_attn_rows > 0) {
    CKC(A.alloc(&hd->f_opart, hd->f_attn_rows * 128));
    CKC(A.alloc(&hd->f_mpart, hd->f_attn_rows));
    CKC(A.alloc(&hd->f_lpart, hd->f_attn_rows));
  }
  const size_t lm_parts = (size_t)(V + 127) / 128;
  CKC(A.alloc(&hd->lm_val, lm_parts * Mx));
  CKC(A.alloc(&hd->lm_idx, lm_parts * Mx));
  CKC(A.alloc(&hd->kv_seq, (size_t)d.max_batch + 1));
  CKC(A.alloc(&hd->dev_err, 1));
  CKC(cudaMemset(hd->dev_err, 0, sizeof(int)));
  CKC(cudaDeviceSynchronize());
#undef CKC
  *out = hd;
  return DFLASH_OK;
}

int dflash_destroy(void* handle) {
  if (!handle) return fail(DFLASH_ERR_INVALID, "NULL handle");
  Handle* hd = static_cast<Handle*>(handle);
  cudaSetDevice(hd->device);
  cudaDeviceSynchronize();
  hd->arena.release();
  delete hd;
  return DFLASH_OK;
}

int dflash_device_status(void* handle, void* stream) {
  if (!handle) return fail(DFLASH_ERR_INVALID, "NULL handle");
  Handle* hd = static_cast<Handle*>(handle);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int v = 0;
  CK(cudaMemcpyAsync(&v, hd->dev_err, sizeof(int), cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  if (v != 0) {
    CK(cudaMemsetAsync(hd->dev_err, 0, sizeof(int), st));
    CK(cudaStreamSynchronize(st));
    return fail(DFLASH_ERR_DEVICE, "device wait limit reached (code %d)", v);
  }
  return DFLASH_OK;
}

int dflash_probe_bounded_wait(void* handle, uint32_t polls, void* stream) {
  if (!handle) return fail(DFLASH_ERR_INVALID, "NULL handle");
  Handle* hd = static_cast<Handle*>(handle);
  CK(cudaSetDevice(hd->device));
  CK(bounded_wait_probe_launch(polls, hd->dev_err, static_cast<cudaStream_t>(stream)));
  return DFLASH_OK;
}

int dflash_forward(void* handle, const DFlashForwardArgs* a, void* stream) {
  if (!handle || !a) return fail(DFLASH_ERR_INVALID, "NULL handle or args");
  Handle* hd = static_cast<Handle*>(handle);
  const DFlashDims& d = hd->d;
  const int H = d.hidden_size, I = d.intermediate_size, NQ = d.num_attention_heads,
            NKV = d.num_key_value_heads, F = d.num_target_features;
  const int b = a->batch, B = a->block, nl = a->num_layers;
  if (b < 1 || b > d.max_batch) return fail(DFLASH_ERR_INVALID, "batch %d outside [1, %d]", b, d.max_batch);
  if (B < 2 || B > d.max_block) return fail(DFLASH_ERR_INVALID, "block %d outside [2, %d]", B, d.max_block);
  if (nl < 1 || nl > d.num_hidden_layers)
    return fail(DFLASH_ERR_INVALID, "num_layers %d outside [1, %d]", nl, d.num_hidden_layers);
  // per-sequence context rows, packed in sequence order
  KvMap m{};
  m.nseq = b;
  m.seq = hd->kv_seq;
  std::vector<KvSeq> sq(b + 1, KvSeq{});
  int cmax = 0;
  for (int s = 0; s < b; ++s) {
    const int c = a->ctx_lens ? a->ctx_lens[s] : a->ctx_len;
    if (c < 0 || c > d.max_ctx)
      return fail(DFLASH_ERR_INVALID, "ctx_len %d of sequence %d outside [0, %d]", c, s, d.max_ctx);
    sq[s + 1].ctx_start = sq[s].ctx_start + c;
    cmax = std::max(cmax, c);
  }
  const int Ctot = sq[b].ctx_start;
  if (Ctot > ctx_rows_capacity(d))
    return fail(DFLASH_ERR_INVALID, "%d context rows above the capacity %d", Ctot, ctx_rows_capacity(d));
  if (!a->noise || (Ctot > 0 && !a->target_hidden && !a->target_layers))
    return fail(DFLASH_ERR_INVALID, "noise / target_hidden must not be NULL");
  TcSources fc_src{};
  if (Ctot > 0) {
    if (a->target_layers) {
      if (F > kTcMaxSrc) return fail(DFLASH_ERR_INVALID, "target_layers: %d features above %d", F, kTcMaxSrc);
      const long long ld = a->target_layers_ld ? a->target_layers_ld : H;
      if (ld < H || ld % 8) return fail(DFLASH_ERR_INVALID, "target_layers_ld %lld: not >= %d and a multiple of 8", ld, H);
      for (int f = 0; f < F; ++f) {
        if (!a->target_layers[f] || (reinterpret_cast<uintptr_t>(a->target_layers[f]) & 15))
          return fail(DFLASH_ERR_INVALID, "target_layers[%d] is NULL or not 16-byte aligned", f);
        fc_src.ptr[f] = a->target_layers[f];
        fc_src.ld[f] = ld;
      }
      fc_src.n = F;
      fc_src.cols = H;
    } else {
      fc_src.ptr[0] = a->target_hidden;
      fc_src.ld[0] = (long long)F * H;
      fc_src.n = 1;
      fc_src.cols = F * H;
    }
  }
  if (a->target_tokens && (!a->acc_len || !a->correction))
    return fail(DFLASH_ERR_INVALID, "acc_len and correction are required with target_tokens");
  if (hd->f32) return forward_f32(hd, a, sq, static_cast<cudaStream_t>(stream));
  const int top_k = a->anchor_top_k ? a->anchor_top_k : 8;
  const long long anchor_ld = a->anchor_logits_ld ? a->anchor_logits_ld : d.vocab_size;
  if (a->anchor_logits && (top_k < 1 || top_k > kSaMaxK || top_k > d.vocab_size))
    return fail(DFLASH_ERR_INVALID, "anchor_top_k %d outside [1, %d]", top_k, kSaMaxK);
  if (a->anchor_logits && anchor_ld < d.vocab_size)
    return fail(DFLASH_ERR_INVALID, "anchor_logits_ld %lld below vocab_size %d", anchor_ld, d.vocab_size);
  Cache* cc = static_cast<Cache*>(a->cache);
  if (cc && cc->owner != hd) return fail(DFLASH_ERR_INVALID, "the cache belongs to another handle");
  if (cc && b > cc->max_batch)
    return fail(DFLASH_ERR_INVALID, "batch %d above the cache's %d sequences", b, cc->max_batch);
  if (cc && nl != cc->layers)
    return fail(DFLASH_ERR_INVALID, "num_layers %d differs from the cache's %d layers", nl, cc->layers);
  if (a->cache_seqs && !cc) return fail(DFLASH_ERR_INVALID, "cache_seqs needs a cache");
  std::vector<int> cseq(b);
  for (int s = 0; s < b; ++s) cseq[s] = a->cache_seqs ? a->cache_seqs[s] : s;
  if (a->cache_seqs) {
    std::vector<char> seen(cc->max_batch, 0);
    for (int s = 0; s < b; ++s) {
      if (cseq[s] < 0 || cseq[s] >= cc->max_batch || seen[cseq[s]])
        return fail(DFLASH_ERR_INVALID, "cache_seqs[%d] = %d: not a distinct sequence of [0, %d)", s, cseq[s],
                    cc->max_batch);
      seen[cseq[s]] = 1;
    }
  }
  std::lock_guard<std::mutex> lock(hd->mu);
  std::unique_lock<std::mutex> cache_lock;
  if (cc) cache_lock = std::unique_lock<std::mutex>(cc->mu);

  // where this step's K/V rows go and which rows attention reads
  __half *Kbase, *Vbase;
  size_t layer_stride;
  std::vector<SeqState> next;
  if (cc) {
    // update_and_fetch (dflash.py:168-193): append C_s + B rows, then keep
    // the sink and the last window rows when the list outgrows them
    m.sink = cc->sink; m.ring = cc->ring; m.slots = cc->slots;
    next.resize(b);
    for (int s = 0; s < b; ++s) {
      const SeqState s0 = cc->at(0, cseq[s]);
      for (int l = 1; l < nl; ++l)
        if (!(cc->at(l, cseq[s]) == s0))
          return fail(DFLASH_ERR_INVALID,
                      "cache layers hold different rows for sequence %d (trim every layer alike)", s);
      const int app = sq[s + 1].ctx_start - sq[s].ctx_start + B;
      const int to_sink = s0.hl < cc->sink ? std::min(app, cc->sink - s0.hl) : 0;
      SeqState n1 = s0;
      n1.hl = s0.hl + to_sink;
      n1.rl = s0.rl + app - to_sink;
      if (n1.rl > cc->ring)
        return fail(DFLASH_ERR_INVALID, "cache full: sequence %d would hold %d rows, capacity %d", s,
                    n1.hl + n1.rl, cc->slots);
      if (cc->evict && n1.hl + n1.rl > cc->sink_size + cc->window_size) {
        n1.rs = (s0.rs + n1.rl - cc->window_size) % cc->ring;
        n1.rl = cc->window_size;
      }
      n1.offset = s0.offset + app;
      sq[s].n0 = s0.hl + s0.rl;
      sq[s].rs_pre = s0.rs;
      sq[s].rs_post = n1.rs;
      sq[s].n_att = n1.hl + n1.rl;
      sq[s].pos0 = s0.offset;
      sq[s].cseq = cseq[s];
      next[s] = n1;
    }
    Kbase = cc->K; Vbase = cc->V;
    layer_stride = cc->layer_stride;
  } else {
    // cache=None: the step's own C_s + B rows, nothing kept
    m.sink = 0; m.ring = m.slots = cmax + B;
    for (int s = 0; s < b; ++s) {
      const int off = a->rope_offsets ? a->rope_offsets[s] : a->rope_offset;
      if (off < 0) return fail(DFLASH_ERR_INVALID, "rope offsets must be >= 0");
      sq[s].n0 = 0; sq[s].rs_pre = 0; sq[s].rs_post = 0;
      sq[s].n_att = sq[s + 1].ctx_start - sq[s].ctx_start + B;
      sq[s].pos0 = off;
      sq[s].cseq = s;
    }
    Kbase = hd->K; Vbase = hd->V;
    if ((size_t)b * m.slots > hd->stateless_rows)
      return fail(DFLASH_ERR_INVALID, "stateless step needs %zu K/V rows (batch * (longest context + block)), "
                  "capacity %zu", (size_t)b * m.slots, hd->stateless_rows);
    layer_stride = (size_t)b * NKV * m.slots * 128;
  }
  int kvmax = 0;
  for (int s = 0; s < b; ++s) kvmax = std::max(kvmax, sq[s].n_att);

  CK(cudaSetDevice(hd->device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int M = b * B;
  const int G = NQ / NKV;
  const bool dense = M > kW8Rows;
  const bool lm_dense = dense;   // the lm_head as a dense tcgen05 GEMM above kW8Rows rows
  if (dense && !hd->dense) return fail(DFLASH_ERR_INVALID, "%d block rows above %d", M, kW8Rows);
  const bool timing = a->phase_events && a->n_phase_events >= DFLASH_PHASES;
  auto mark = [&](int k) -> cudaError_t {
    return timing ? cudaEventRecord(static_cast<cudaEvent_t>(a->phase_events[k]), st) : cudaSuccess;
  };
  int launches = 0;

  CK(mark(0));
  CK(rope_table_map_launch(m, sq.data(), B, hd->inv_freq, hd->rope, st));
  if (b + 1 > kKvChunk) launches += (b + kKvChunk) / kKvChunk;   // kv_upload launches
  if (a->anchor_logits) {
    SaParams sp{};
    sp.logits = a->anchor_logits; sp.logits_bf16 = a->anchor_logits_bf16 != 0;
    sp.V = d.vocab_size; sp.ld = anchor_ld; sp.k = top_k;
    sp.E = hd->lm_tiles; sp.H = H; sp.out = hd->anchor; sp.out_ld = H;
    sp.cand_v = hd->sa_cand_v; sp.cand_i = hd->sa_cand_i; sp.counter = hd->sa_cnt;
    CK(soft_anchor_launch(sp, b, true, hd->num_sms, st));
    launches += 1;
  }
  CK(init_h_launch(reinterpret_cast<const __nv_bfloat16*>(a->noise), M, H, hd->h, hd->hstat,
                   hd->layers[0].in_norm, hd->hmax, a->anchor_logits ? hd->anchor : nullptr, B, st));
  launches += 2;
  CK(mark(1));

  if (Ctot > 0) {
    TcParams fp{};
    fp.tail_part = hd->tc_part; fp.tail_cnt = hd->tc_cnt; fp.tail_cap = hd->tc_cap;
    fp.M = Ctot; fp.N = H; fp.K = F * H; fp.err = hd->dev_err;
    // hidden_norm (dflash.py:392): the fc epilogue stores the fp32 rows with
    // per-256-column sums of squares; ctx_norm rounds the normalised rows to
    // f16 (11 mantissa bits, and no overflow once normalised), the context
    // K|V GEMM's A operand
    fp.out_f32 = hd->ctx_raw; fp.sumsq_part = hd->ctx_part;
    CK(tc_gemm_launch_src(fc_src, hd->fc, true, kTcFc, fp, st));
    CK(mark(2));
    CK(ctx_norm_launch(hd->ctx_raw, hd->ctx_part, H / 256, Ctot, H, hd->hidden_norm, d.rms_norm_eps, hd->ctx_n,
                       st));
    CK(mark(3));
    TcParams kp{};
    kp.tail_part = hd->tc_part; kp.tail_cnt = hd->tc_cnt; kp.tail_cap = hd->tc_cap;
    kp.M = Ctot; kp.N = nl * 2 * NKV * 128; kp.K = H; kp.err = hd->dev_err;
    kp.scale = hd->s_kv_ctx; kp.k_norm = hd->k_norm_all; kp.rope = hd->rope;
    kp.k_out = Kbase; kp.v_out = Vbase; kp.layer_stride = layer_stride;
    kp.nkv = NKV; kp.eps = d.rms_norm_eps; kp.kv = m;
    CK(tc_gemm_launch(hd->ctx_n, hd->w_kv_ctx, false, kTcCtxKV, kp, st));
    CK(mark(4));
    launches += 3;   // fc, hidden_norm, context K|V
  } else {
    CK(mark(2));
    CK(mark(3));
    CK(mark(4));
  }

  int chunk, splits;
  attn_pick_split(b, NKV, kvmax, hd->num_sms, G * B, &chunk, &splits);
  if ((size_t)b * NKV * splits * G * B > hd->attn_part_rows)
    return fail(DFLASH_ERR_INVALID, "attention workspace too small");
  int hparts = 1;
  const float attn_scale_log2 = (float)(1.0 / std::sqrt(128.0) * 1.4426950408889634);
  // dense block path: every projection a persistent tcgen05 GEMM over the
  // exact f16 weight copies, the RMSNorms as separate f16 row kernels
  for (int l = 0; dense && l < nl; ++l) {
    const Layer& ly = hd->layers[l];
    __half* Kl = Kbase + l * layer_stride;
    __half* Vl = Vbase + l * layer_stride;
    CK(ctx_norm_launch(hd->h, hd->hstat, hparts, M, H, ly.in_norm, d.rms_norm_eps, hd->xa, st));
    TcParams qp{};
    qp.tail_part = hd->tc_part; qp.tail_cnt = hd->tc_cnt; qp.tail_cap = hd->tc_cap;
    qp.M = M; qp.N = (NQ + 2 * NKV) * 128; qp.K = H; qp.err = hd->dev_err;
    qp.scale = ly.s_qkv; qp.q_norm = ly.q_norm; qp.k_norm = hd->k_norm_all + l * 128;
    qp.rope = hd->rope; qp.rope_row0 = Ctot; qp.eps = d.rms_norm_eps;
    qp.q_out = hd->Q; qp.k_out = Kl; qp.v_out = Vl;
    qp.nkv = NKV; qp.n_q_heads = NQ; qp.block = B; qp.kv = m;
    CK(tc_gemm_launch(hd->xa, ly.dw_qkv, false, kTcBlkQKV, qp, st));
    AttnParams ap{};
    ap.q = hd->Q; ap.k = Kl; ap.v = Vl; ap.nq = NQ; ap.nkv = NKV; ap.block = B; ap.kv_len = kvmax;
    ap.kv_cap = m.slots; ap.chunk = chunk; ap.splits = splits; ap.opart = hd->opart;
    ap.mpart = hd->mpart; ap.lpart = hd->lpart; ap.scale_log2 = attn_scale_log2;
    ap.kv = m; ap.kv_seqs = cc ? cc->max_batch : b; ap.err = hd->dev_err;
    CK(attn_tc_launch(ap, b, hd->attn_out, st));
    TcParams op{};
    op.tail_part = hd->tc_part; op.tail_cnt = hd->tc_cnt; op.tail_cap = hd->tc_cap;
    op.M = M; op.N = H; op.K = NQ * 128; op.err = hd->dev_err;
    op.scale = ly.s_o; op.h = hd->h; op.sumsq_part = hd->hstat;
    CK(tc_gemm_launch(hd->attn_out, ly.dw_o, false, kTcResid, op, st));
    hparts = H / 256;
    CK(ctx_norm_launch(hd->h, hd->hstat, hparts, M, H, ly.post_norm, d.rms_norm_eps, hd->xa, st));
    TcParams gp{};
    gp.tail_part = hd->tc_part; gp.tail_cnt = hd->tc_cnt; gp.tail_cap = hd->tc_cap;
    gp.M = M; gp.N = 2 * I; gp.K = H; gp.err = hd->dev_err; gp.scale = ly.ds_gu; gp.act = hd->act;
    CK(tc_gemm_launch(hd->xa, ly.dw_gu, false, kTcSilu, gp, st));
    TcParams dp{};
    dp.tail_part = hd->tc_part; dp.tail_cnt = hd->tc_cnt; dp.tail_cap = hd->tc_cap;
    dp.M = M; dp.N = H; dp.K = I; dp.err = hd->dev_err;
    dp.scale = ly.s_d; dp.h = hd->h; dp.sumsq_part = hd->hstat;
    CK(tc_gemm_launch(hd->act, ly.dw_d, false, kTcResid, dp, st));
    launches += 7 + (splits > 1);  // 2 norms, q|k|v, attention (+ combine), o, gate|up, down
  }
  for (int l = 0; !dense && l < nl; ++l) {
    const Layer& ly = hd->layers[l];
    __half* Kl = Kbase + l * layer_stride;
    __half* Vl = Vbase + l * layer_stride;
    // q | k | v of the block rows: input RMSNorm fused into the activation load
    CK(rmsnorm_limbs_launch(hd->h, hd->hstat, hd->hmax, hparts, M, H, ly.in_norm, d.rms_norm_eps,
                            hd->xl, hd->xs, st));
    W8Params p{};
    p.scale = ly.s_qkv; p.N = (NQ + 2 * NKV) * 128; p.K = H; p.M = M;
    p.xl = hd->xl; p.xscale = hd->xs; p.eps = d.rms_norm_eps;
    p.q_out = hd->Q; p.k_out = Kl; p.v_out = Vl; p.q_norm = ly.q_norm; p.k_norm = hd->k_norm_all + l * 128;
    p.rope = hd->rope; p.n_q_heads = NQ; p.n_kv_heads = NKV; p.block = B; p.rope_blk0 = Ctot;
    p.kv = m;
    CK(w8tc_launch(ly.w_qkv, p, kQKV, hd->dev_err, hd->w8_part, hd->w8_part_floats, hd->w8_cnt, hd->num_sms, st));
    // attention over each sequence's stored rows
    AttnParams ap{};
    ap.q = hd->Q; ap.k = Kl; ap.v = Vl; ap.nq = NQ; ap.nkv = NKV; ap.block = B; ap.kv_len = kvmax;
    ap.kv_cap = m.slots; ap.chunk = chunk; ap.splits = splits; ap.opart = hd->opart;
    ap.mpart = hd->mpart; ap.lpart = hd->lpart;
    ap.scale_log2 = attn_scale_log2;
    ap.normrope = 0;
    ap.kv = m; ap.kv_seqs = cc ? cc->max_batch : b;
    ap.omax = hd->amax;
    ap.err = hd->dev_err;
    // with several KV splits the merge writes the o-projection's limbs itself
    AttnLimbOut lo{hd->xl, hd->xs, M, false};
    CK(attn_tc_launch(ap, b, hd->attn_out, st, &lo));
    // o_proj + residual
    W8Params o{};
    if (!lo.done) CK(w8_limbs_launch(hd->attn_out, M, NQ * 128, hd->amax, NQ, hd->xl, hd->xs, st));
    o.scale = ly.s_o; o.N = H; o.K = NQ * 128; o.M = M; o.xl = hd->xl; o.xscale = hd->xs;
    o.h_out = hd->h; o.hstat_out = hd->hstat; o.hmax_out = hd->hmax; o.next_norm = ly.post_norm;
    CK(w8tc_launch(ly.w_o, o, kResid, hd->dev_err, hd->w8_part, hd->w8_part_floats, hd->w8_cnt, hd->num_sms, st));
    hparts = H / 128;
    // gate|up with post-attention RMSNorm fused, silu(g)*u epilogue
    CK(rmsnorm_limbs_launch(hd->h, hd->hstat, hd->hmax, hparts, M, H, ly.post_norm, d.rms_norm_eps,
                            hd->xl, hd->xs, st));
    W8Params gu{};
    gu.scale = ly.s_gu; gu.N = 2 * I; gu.K = H; gu.M = M;
    gu.xl = hd->xl; gu.xscale = hd->xs; gu.act = hd->act_w8; gu.amax_out = hd->amax;
    CK(w8tc_launch(ly.w_gu, gu, kSiluMul, hd->dev_err, hd->w8_part, hd->w8_part_floats, hd->w8_cnt, hd->num_sms, st));
    // down + residual
    W8Params dn{};
    CK(w8_limbs_launch(hd->act_w8, M, I, hd->amax, 2 * I / 128, hd->xl, hd->xs, st));
    dn.scale = ly.s_d; dn.N = H; dn.K = I; dn.M = M; dn.xl = hd->xl; dn.xscale = hd->xs;
    dn.h_out = hd->h; dn.hstat_out = hd->hstat;
    if (l + 1 < nl) {  // the next layer's input RMSNorm reads h
      dn.hmax_out = hd->hmax;
      dn.next_norm = hd->layers[l + 1].in_norm;
    }
    CK(w8tc_launch(ly.w_d, dn, kResid, hd->dev_err, hd->w8_part, hd->w8_part_floats, hd->w8_cnt, hd->num_sms, st));
    // 2 norms + limbs of the SiLU output, qkv, attention, merge and/or limbs of its output,
    // o, gate|up, down
    launches += 8 + (splits > 1) + (lo.done ? 0 : 1);
  }
  CK(mark(5));
  // dense path: the lm_head reads only rows 1..B-1 of every block, packed
  CK(final_norm_launch(hd->h, hd->hstat, hparts, M, H, hd->norm, d.rms_norm_eps, hd->hn,
                       a->out_hidden, a->out_hidden_fp32 != 0, st, B, lm_dense ? 1 : 0));
  launches += 1;
  CK(mark(6));
  if (a->out_tokens || a->target_tokens) {
    LmParams lp{};
    lp.hn = hd->hn; lp.V = d.vocab_size; lp.H = H; lp.M = M;
    lp.best_val = hd->lm_val; lp.best_idx = hd->lm_idx;
    int grid = 0;
    if (lm_dense) {
      TcParams tp{};
    tp.tail_part = hd->tc_part; tp.tail_cnt = hd->tc_cnt; tp.tail_cap = hd->tc_cap;
      tp.M = b * (B - 1); tp.N = (d.vocab_size + 255) / 256 * 256; tp.K = H; tp.err = hd->dev_err;
      tp.V = d.vocab_size; tp.best_val = hd->lm_val; tp.best_idx = hd->lm_idx;
      CK(tc_gemm_launch(hd->hn, hd->lm_tiles, true, kTcArgmax, tp, st));
      grid = tp.N / 256;
    } else {
      CK(lm_argmax_launch(lp, hd->lm_tiles, hd->num_sms, hd->dev_err, &grid, st));
    }
    CK(argmax_accept_launch(hd->lm_val, hd->lm_idx, grid, lm_dense ? b * (B - 1) : M, B, b, a->out_tokens,
                            a->target_tokens, a->acc_len, a->correction, st, lm_dense ? 1 : 0));
    launches += 2;
  }
  CK(mark(7));
  if (cc)
    for (int l = 0; l < nl; ++l)
      for (int s = 0; s < b; ++s) cc->at(l, cseq[s]) = next[s];
  hd->last_launches = launches;
  return DFLASH_OK;
}

// ---------------------------------------------------------------- KV cache
int dflash_cache_create(void* handle, int num_layers, int max_batch, int sink_size, int window_size,
                        int max_len, void** out) {
  if (!handle || !out) return fail(DFLASH_ERR_INVALID, "NULL handle or output");
  Handle* hd = static_cast<Handle*>(handle);
  const DFlashDims& d = hd->d;
  if (num_layers < 1 || num_layers > d.num_hidden_layers)
    return fail(DFLASH_ERR_INVALID, "num_layers %d outside [1, %d]", num_layers, d.num_hidden_layers);
  if (max_batch < 1 || max_batch > d.max_batch)
    return fail(DFLASH_ERR_INVALID, "max_batch %d outside [1, %d]", max_batch, d.max_batch);
  Cache* c = new Cache();
  c->owner = hd;
  c->device = hd->device;
  c->nkv = d.num_key_value_heads;
  c->layers = num_layers;
  c->max_batch = max_batch;
  c->sink_size = sink_size;
  c->window_size = window_size;
  c->evict = sink_size > 0 && window_size > 0;
  if (c->evict) {
    // before eviction a step holds at most window + (max_ctx + max_block) ring rows
    c->sink = sink_size;
    c->ring = window_size + d.max_ctx + d.max_block;
  } else {
    if (max_len < 1) {
      delete c;
      return fail(DFLASH_ERR_INVALID, "a cache without eviction needs max_len >= 1 (got %d)", max_len);
    }
    c->sink = 0;
    c->ring = max_len;
  }
  c->slots = c->sink + c->ring;
  c->layer_stride = (size_t)max_batch * d.num_key_value_heads * c->slots * 128;
  c->st.assign((size_t)num_layers * max_batch, SeqState{});
  const size_t elems = c->layer_stride * num_layers;
  cudaError_t e = cudaSetDevice(hd->device);
  if (e == cudaSuccess) e = cudaMalloc(&c->K, elems * 2);
  if (e == cudaSuccess) e = cudaMalloc(&c->V, elems * 2);
  if (e != cudaSuccess) {
    if (c->K) cudaFree(c->K);
    delete c;
    return fail(e == cudaErrorMemoryAllocation ? DFLASH_ERR_OOM : DFLASH_ERR_CUDA,
                "cache allocation of 2 x %zu bytes: %s", elems * 2, cudaGetErrorString(e));
  }
  *out = c;
  return DFLASH_OK;
}

int dflash_cache_trim(void* cache, int layer, int n) {
  if (!cache) return fail(DFLASH_ERR_INVALID, "NULL cache");
  Cache* c = static_cast<Cache*>(cache);
  if (layer >= c->layers) return fail(DFLASH_ERR_INVALID, "layer %d outside [0, %d)", layer, c->layers);
  if (n <= 0) return DFLASH_OK;
  std::lock_guard<std::mutex> lock(c->mu);
  const int l0 = layer < 0 ? 0 : layer, l1 = layer < 0 ? c->layers : layer + 1;
  for (int l = l0; l < l1; ++l)
    for (int s = 0; s < c->max_batch; ++s) trim_state(c->at(l, s), n);
  return DFLASH_OK;
}

int dflash_cache_trim_seqs(void* cache, int layer, const int32_t* seqs, const int32_t* counts, int count) {
  if (!cache || (count > 0 && (!seqs || !counts))) return fail(DFLASH_ERR_INVALID, "NULL argument");
  Cache* c = static_cast<Cache*>(cache);
  if (layer >= c->layers) return fail(DFLASH_ERR_INVALID, "layer %d outside [0, %d)", layer, c->layers);
  for (int i = 0; i < count; ++i)
    if (seqs[i] < 0 || seqs[i] >= c->max_batch || counts[i] < 0)
      return fail(DFLASH_ERR_INVALID, "trim entry %d: sequence %d / count %d", i, seqs[i], counts[i]);
  std::lock_guard<std::mutex> lock(c->mu);
  const int l0 = layer < 0 ? 0 : layer, l1 = layer < 0 ? c->layers : layer + 1;
  for (int l = l0; l < l1; ++l)
    for (int i = 0; i < count; ++i) trim_state(c->at(l, seqs[i]), counts[i]);
  return DFLASH_OK;
}

int dflash_cache_reset(void* cache) {
  if (!cache) return fail(DFLASH_ERR_INVALID, "NULL cache");
  Cache* c = static_cast<Cache*>(cache);
  std::lock_guard<std::mutex> lock(c->mu);
  for (auto& q : c->st) q = SeqState{};
  return DFLASH_OK;
}

int dflash_cache_reset_seqs(void* cache, const int32_t* seqs, int count) {
  if (!cache || (count > 0 && !seqs)) return fail(DFLASH_ERR_INVALID, "NULL argument");
  Cache* c = static_cast<Cache*>(cache);
  for (int i = 0; i < count; ++i)
    if (seqs[i] < 0 || seqs[i] >= c->max_batch)
      return fail(DFLASH_ERR_INVALID, "sequence %d outside [0, %d)", seqs[i], c->max_batch);
  std::lock_guard<std::mutex> lock(c->mu);
  for (int l = 0; l < c->layers; ++l)
    for (int i = 0; i < count; ++i) c->at(l, seqs[i]) = SeqState{};
  return DFLASH_OK;
}

int dflash_cache_state(void* cache, int layer, int seq, int32_t* offset, int32_t* length) {
  if (!cache) return fail(DFLASH_ERR_INVALID, "NULL cache");
  Cache* c = static_cast<Cache*>(cache);
  if (layer < 0 || layer >= c->layers || seq < 0 || seq >= c->max_batch)
    return fail(DFLASH_ERR_INVALID, "layer %d / sequence %d out of range", layer, seq);
  std::lock_guard<std::mutex> lock(c->mu);
  const SeqState& q = c->at(layer, seq);
  if (offset) *offset = q.offset;
  if (length) *length = q.hl + q.rl;
  return DFLASH_OK;
}

int dflash_cache_read(void* cache, int layer, int seq, uint16_t* keys, uint16_t* values, void* stream) {
  if (!cache) return fail(DFLASH_ERR_INVALID, "NULL cache");
  Cache* c = static_cast<Cache*>(cache);
  if (layer < 0 || layer >= c->layers || seq < 0 || seq >= c->max_batch)
    return fail(DFLASH_ERR_INVALID, "layer %d / sequence %d out of range", layer, seq);
  std::lock_guard<std::mutex> lock(c->mu);
  const SeqState q = c->at(layer, seq);
  const int NKV = c->nkv;
  const int len = q.hl + q.rl;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CK(cudaSetDevice(c->device));
  // logical rows: sink slots [0, hl), then ring rows from rs (wrapping once)
  const int first = std::min(q.rl, c->ring - q.rs);
  const struct { int dst, src, n; } runs[3] = {
      {0, 0, q.hl}, {q.hl, c->sink + q.rs, first}, {q.hl + first, c->sink, q.rl - first}};
  for (int which = 0; which < 2; ++which) {
    uint16_t* dst = which ? values : keys;
    if (!dst) continue;
    const __half* base = (which ? c->V : c->K) + layer * c->layer_stride +
                         (size_t)seq * NKV * c->slots * 128;
    for (int h = 0; h < NKV; ++h)
      for (const auto& r : runs)
        if (r.n > 0)
          CK(cudaMemcpyAsync(dst + ((size_t)h * len + r.dst) * 128,
                             base + ((size_t)h * c->slots + r.src) * 128, (size_t)r.n * 128 * 2,
                             cudaMemcpyDeviceToDevice, st));
  }
  return DFLASH_OK;
}

int dflash_cache_destroy(void* cache) {
  if (!cache) return fail(DFLASH_ERR_INVALID, "NULL cache");
  Cache* c = static_cast<Cache*>(cache);
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  cudaFree(c->K);
  cudaFree(c->V);
  delete c;
  return DFLASH_OK;
}

int dflash_last_launch_count(void* handle) {
  if (!handle) return fail(DFLASH_ERR_INVALID, "NULL handle");
  return static_cast<Handle*>(handle)->last_launches;
}

int dflash_accept(const int32_t* draft, const int32_t* target, int batch, int block,
                  int32_t* acc_len, int32_t* correction, void* stream) {
  if (!draft || !target || !acc_len || !correction) return fail(DFLASH_ERR_INVALID, "NULL pointer");
  if (batch < 1 || block < 2) return fail(DFLASH_ERR_INVALID, "batch >= 1 and block >= 2 required");
  CK(accept_launch(draft, target, batch, block, acc_len, correction, static_cast<cudaStream_t>(stream)));
  return DFLASH_OK;
}

int dflash_quantize_q8(const float* w, int oc, int ic, int8_t* q, uint16_t* s, void* stream) {
  if (!w || !q || !s) return fail(DFLASH_ERR_INVALID, "NULL pointer");
  if (oc < 1 || ic < 1) return fail(DFLASH_ERR_INVALID, "oc and ic must be positive");
  CK(quantize_q8_launch(w, oc, ic, q, reinterpret_cast<__half*>(s), static_cast<cudaStream_t>(stream)));
  return DFLASH_OK;
}

// ---------------------------------------------------------------- kernel-level
int dflash_w8_linear(const int8_t* q, const uint16_t* s, int N, int K, const uint16_t* x, int M,
                     uint16_t* y, void* stream) {
  if (!q || !s || !x || !y) return fail(DFLASH_ERR_INVALID, "NULL pointer");
  if (N % 128 || K % 128 || M < 1 || M > 64)
    return fail(DFLASH_ERR_INVALID, "need N %% 128 == 0, K %% 128 == 0, 1 <= M <= 64");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0, sms = 148;
  CK(cudaGetDevice(&dev));
  CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  float* sp = nullptr;
  int* err = nullptr;
  CK(cudaMallocAsync(&sp, (size_t)N * 4, st));
  CK(cudaMallocAsync(&err, sizeof(int), st));
  CK(cudaMemsetAsync(err, 0, sizeof(int), st));
  CK(w8_scale_launch(reinterpret_cast<const __half*>(s), N, sp, 1 << 30, 0, 0, st));
  int8_t* wt = nullptr;
  CK(cudaMallocAsync(&wt, (size_t)N * K, st));
  CK(w8_tilepack_launch(q, N, K, wt, 1 << 30, 0, 0, st));
  int8_t* xl = nullptr;
  float* xs = nullptr;
  CK(cudaMallocAsync(&xl, (size_t)3 * 64 * K, st));
  CK(cudaMallocAsync(&xs, 64 * sizeof(float), st));
  CK(w8_limbs_launch(reinterpret_cast<const __half*>(x), M, K, nullptr, 0, xl, xs, st));
  W8Params p{};
  p.scale = sp; p.N = N; p.K = K; p.M = M;
  p.xl = xl; p.xscale = xs; p.y = reinterpret_cast<__half*>(y);
  const size_t pf = w8tc_part_floats(N, K, M, sms);
  float* part = nullptr;
  int* cnt = nullptr;
  CK(cudaMallocAsync(&part, (pf > 0 ? pf : 1) * sizeof(float), st));
  CK(cudaMallocAsync(&cnt, (size_t)(N / 128) * sizeof(int), st));
  CK(cudaMemsetAsync(cnt, 0, (size_t)(N / 128) * sizeof(int), st));
  cudaError_t e = w8tc_launch(wt, p, kStore, err, part, pf, cnt, sms, st);
  int hv = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&hv, err, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  for (void* ptr : {(void*)sp, (void*)xl, (void*)xs, (void*)wt, (void*)part, (void*)cnt, (void*)err}) {
    const cudaError_t f = cudaFreeAsync(ptr, st);
    if (e == cudaSuccess) e = f;
  }
  CK(e);
  if (hv) return fail(DFLASH_ERR_DEVICE, "W8A16 kernel gave up on a bounded wait (code %d)", hv);
  return DFLASH_OK;
}

int dflash_tc_gemm(const uint16_t* A, const uint16_t* B, int M, int N, int K, int ab_bf16, float* D,
                   void* stream) {
  if (!A || !B || !D) return fail(DFLASH_ERR_INVALID, "NULL pointer");
  if (M < 1 || N % 256 || K % 64 || K < 64)
    return fail(DFLASH_ERR_INVALID, "need M >= 1, N %% 256 == 0, K %% 64 == 0");
  TcParams p{};
  p.M = M; p.N = N; p.K = K; p.out_f32 = D;
  int* err = nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CK(cudaMallocAsync(&err, sizeof(int), st));
  CK(cudaMemsetAsync(err, 0, sizeof(int), st));
  p.err = err;
  // tail-split workspace, as the draft forward gives its GEMMs
  int dev = 0, sms = 148;
  CK(cudaGetDevice(&dev));
  CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  p.tail_cap = 4 * sms;
  CK(cudaMallocAsync(&p.tail_part, (size_t)p.tail_cap * 128 * 256 * sizeof(float), st));
  CK(cudaMallocAsync(&p.tail_cnt, (size_t)sms * sizeof(int), st));
  CK(cudaMemsetAsync(p.tail_cnt, 0, (size_t)sms * sizeof(int), st));
  cudaError_t e = tc_gemm_launch(A, B, ab_bf16 != 0, kTcStoreF32, p, st);
  int hv = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&hv, err, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  for (void* ptr : {(void*)p.tail_part, (void*)p.tail_cnt, (void*)err}) {
    const cudaError_t f = cudaFreeAsync(ptr, st);
    if (e == cudaSuccess) e = f;
  }
  CK(e);
  if (hv) return fail(DFLASH_ERR_DEVICE, "tcgen05 GEMM gave up on a bounded wait (code %d)", hv);
  return DFLASH_OK;
}

size_t dflash_attention_workspace_size(int batch, int nq, int nkv, int block, int kv_len) {
  if (batch < 1 || nkv < 1 || nq % nkv || kv_len < 1) return 0;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int chunk, splits;
  attn_pick_split(batch, nkv, kv_len, sms, (nq / nkv) * block, &chunk, &splits);
  const size_t rows = (size_t)batch * nkv * splits * (nq / nkv) * block;
  const size_t rope_rows = (size_t)kv_len + block;
  return rows * 130 * 4 + rope_rows * 64 * 8 + 64 * 4 + 256;
}

int dflash_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int batch, int nq,
                     int nkv, int block, int kv_len, int normrope, const float* q_norm,
                     const float* k_norm, float rope_theta, int q_pos0, int k_pos0, float eps,
                     uint16_t* out, void* workspace, size_t ws_bytes, void* stream) {
  if (!q || !k || !v || !out || !workspace) return fail(DFLASH_ERR_INVALID, "NULL pointer");
  if (batch < 1 || nkv < 1 || nq % nkv || block < 1 || kv_len < 1)
    return fail(DFLASH_ERR_INVALID, "bad attention shape");
  if ((nq / nkv) * block > 192) return fail(DFLASH_ERR_INVALID, "heads/kv_heads * block must be <= 192");
  if (normrope && (!q_norm || !k_norm || q_pos0 < 0 || k_pos0 < 0))
    return fail(DFLASH_ERR_INVALID, "normrope needs q_norm, k_norm and non-negative positions");
  const size_t need = dflash_attention_workspace_size(batch, nq, nkv, block, kv_len);
  if (ws_bytes < need) return fail(DFLASH_ERR_INVALID, "workspace too small (%zu < %zu)", ws_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0, sms = 148;
  CK(cudaGetDevice(&dev));
  CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  int chunk, splits;
  attn_pick_split(batch, nkv, kv_len, sms, (nq / nkv) * block, &chunk, &splits);
  const size_t rows = (size_t)batch * nkv * splits * (nq / nkv) * block;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  AttnParams p{};
  p.opart = reinterpret_cast<float*>(ws);
  p.mpart = p.opart + rows * 128;
  p.lpart = p.mpart + rows;
  float2* rope = reinterpret_cast<float2*>((reinterpret_cast<uintptr_t>(p.lpart + rows) + 15) & ~uintptr_t(15));
  p.q = reinterpret_cast<const __half*>(q);
  p.k = reinterpret_cast<const __half*>(k);
  p.v = reinterpret_cast<const __half*>(v);
  p.nq = nq; p.nkv = nkv; p.block = block; p.kv_len = kv_len; p.kv_cap = kv_len;
  p.chunk = chunk; p.splits = splits;
  p.scale_log2 = (float)(1.0 / std::sqrt(128.0) * 1.4426950408889634);
  p.normrope = normrope;
  if (normrope) {
    // table rows cover both position ranges: row r <-> position r
    const int maxpos = std::max(q_pos0 + block, k_pos0 + kv_len);
    if ((size_t)maxpos > (size_t)(kv_len + block))
      return fail(DFLASH_ERR_INVALID, "positions must lie below kv_len + block");
    CK(rope_table_launch(0, kv_len + block, rope_theta, rope, st));
    p.q_norm = q_norm; p.k_norm = k_norm; p.rope = rope; p.eps = eps;
    p.q_row0 = q_pos0; p.k_row0 = k_pos0;
  }
  // the tensor-core kernel, or the mma.sync one where Q/K need the fused norm + RoPE
  if (normrope)
    CK(attn_launch(p, batch, reinterpret_cast<__half*>(out), st));
  else
    CK(attn_tc_launch(p, batch, reinterpret_cast<__half*>(out), st));
  return DFLASH_OK;
}

size_t dflash_soft_anchor_workspace_size(int batch) {
  if (batch < 1) return 0;
  return (size_t)batch * kSaMaxCtas * kSaMaxK * 8 + (size_t)batch * sizeof(int) + 256;
}

int dflash_soft_anchor(const void* logits, int logits_bf16, int batch, int V, int64_t ld, int k,
                       const uint16_t* E, int H, uint16_t* out, void* workspace, size_t ws_bytes,
                       void* stream) {
  if (!logits || !E || !out || !workspace) return fail(DFLASH_ERR_INVALID, "NULL pointer");
  if (batch < 1 || V < 1 || ld < V || H < 8 || H % 8)
    return fail(DFLASH_ERR_INVALID, "bad soft anchor shape (batch %d, V %d, ld %lld, H %d)", batch, V,
                (long long)ld, H);
  if (k < 1 || k > kSaMaxK || k > V) return fail(DFLASH_ERR_INVALID, "k %d outside [1, %d]", k, kSaMaxK);
  if ((reinterpret_cast<uintptr_t>(E) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(DFLASH_ERR_INVALID, "E and out must be 16-byte aligned");
  if (ws_bytes < dflash_soft_anchor_workspace_size(batch))
    return fail(DFLASH_ERR_INVALID, "workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0, sms = 148;
  CK(cudaGetDevice(&dev));
  CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const size_t nc = (size_t)batch * kSaMaxCtas * kSaMaxK;
  SaParams p{};
  p.logits = logits; p.logits_bf16 = logits_bf16 != 0; p.V = V; p.ld = ld; p.k = k;
  p.E = E; p.H = H; p.out = reinterpret_cast<__nv_bfloat16*>(out); p.out_ld = H;
  p.cand_v = static_cast<float*>(workspace);
  p.cand_i = reinterpret_cast<int*>(p.cand_v + nc);
  p.counter = p.cand_i + nc;
  CK(cudaMemsetAsync(p.counter, 0, (size_t)batch * sizeof(int), st));
  CK(soft_anchor_launch(p, batch, false, sms, st));
  return DFLASH_OK;
}

// workspace: per-CTA (max, index) partials, the error word, then E repacked
// into the lm_head's 128-row swizzled tiles (1024-byte aligned)
size_t dflash_lm_head_workspace_size(int batch, int block, int V, int H) {
  if (batch < 1 || block < 1 || V < 1 || H < 1) return 0;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return (size_t)sms * batch * block * 8 + 256 + 1024 + lm_pack_bytes(V, H);
}

int dflash_lm_head_argmax(const uint16_t* hn, const uint16_t* E, int batch, int block, int H, int V,
                          int32_t* tokens, const int32_t* target, int32_t* acc_len, int32_t* correction,
                          void* workspace, size_t ws_bytes, void* stream) {
  if (!hn || !E || !workspace) return fail(DFLASH_ERR_INVALID, "NULL pointer");
  if (batch < 1 || block < 2 || batch * block > 64 || H % 64 || V < 1)
    return fail(DFLASH_ERR_INVALID, "bad lm_head shape");
  if (target && (!acc_len || !correction)) return fail(DFLASH_ERR_INVALID, "acc_len/correction required");
  if (ws_bytes < dflash_lm_head_workspace_size(batch, block, V, H))
    return fail(DFLASH_ERR_INVALID, "workspace too small (%zu < %zu)", ws_bytes,
                dflash_lm_head_workspace_size(batch, block, V, H));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0, sms = 148;
  CK(cudaGetDevice(&dev));
  CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int M = batch * block;
  LmParams p{};
  p.hn = reinterpret_cast<const __nv_bfloat16*>(hn);
  p.V = V; p.H = H; p.M = M;
  p.best_val = static_cast<float*>(workspace);
  p.best_idx = reinterpret_cast<int*>(p.best_val + (size_t)sms * M);
  int* err = p.best_idx + (size_t)sms * M;
  uint8_t* et = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(err + 1) + 1023) & ~uintptr_t(1023));
  CK(cudaMemsetAsync(err, 0, sizeof(int), st));
  CK(lm_pack_launch(reinterpret_cast<const __nv_bfloat16*>(E), V, H, et, st));
  int grid = 0;
  CK(lm_argmax_launch(p, et, sms, err, &grid, st));
  CK(argmax_accept_launch(p.best_val, p.best_idx, grid, M, block, batch, tokens, target, acc_len, correction,
                          st));
  return DFLASH_OK;
}

}  // extern "C"

// ---- attention over a static scratch array -------------------------------
//
// dflash_attention_noalloc serves callers that cannot call cudaMalloc: a host
// runtime that has reserved the device's memory for its own pool, or a binding
// that cannot pass a workspace buffer.  It runs the same kernels as
// dflash_attention.  Its workspace is the array below: fixed size, one per
// device that loads the library, held until the process exits.
//
// `g_attn_scratch` is a host-side stand-in for the array.  The device address
// comes from cudaGetSymbolAddress, looked up on every call with the caller's
// device current: after a cudaDeviceReset the library's device code is loaded
// again, possibly at another address, so a cached address could go stale.  The
// lookup is cheap once the code is loaded on the device; the first call on a
// device loads it, so make that first call outside any stream capture.  Calls
// on a device share the array, so calls that overlap on the GPU race.  The
// array keeps the last call's contents.  The partial kernel writes every
// (split, row) partial and the table rows it reads before anything reads them,
// so nothing needs clearing between calls.

static __device__ __align__(256) unsigned char g_attn_scratch[DFLASH_ATTN_STATIC_SCRATCH_BYTES];

namespace {
// device address of g_attn_scratch on the current device
int attn_scratch_ptr(void** out) {
  void* p = nullptr;
  CK(cudaGetSymbolAddress(&p, g_attn_scratch));
  *out = p;
  return DFLASH_OK;
}
}  // namespace

extern "C" int dflash_attention_noalloc(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                        int batch, int nq, int nkv, int block, int kv_len,
                                        int normrope, const float* q_norm, const float* k_norm,
                                        float rope_theta, int q_pos0, int k_pos0, float eps,
                                        uint16_t* out, void* stream) {
  const size_t need = dflash_attention_workspace_size(batch, nq, nkv, block, kv_len);
  if (need > DFLASH_ATTN_STATIC_SCRATCH_BYTES)
    return fail(DFLASH_ERR_INVALID,
                "dflash_attention_noalloc: this shape needs %zu bytes of scratch, more than the "
                "%zu-byte static array; use dflash_attention with a caller workspace",
                need, (size_t)DFLASH_ATTN_STATIC_SCRATCH_BYTES);
  void* scratch = nullptr;
  const int rc = attn_scratch_ptr(&scratch);
  if (rc != DFLASH_OK) return rc;
  return dflash_attention(q, k, v, batch, nq, nkv, block, kv_len, normrope, q_norm, k_norm,
                          rope_theta, q_pos0, k_pos0, eps, out, scratch,
                          DFLASH_ATTN_STATIC_SCRATCH_BYTES, stream);
}
