// Small bandwidth kernels around the projections:
//   rope_table   : (cos, sin) of position * inv_freq for the rows of one
//                  forward (the ANE host precomputes the same tables,
//                  ane_model.py:484-527)
//   init_h       : residual stream h = noise (fp32) and its sum-of-squares
//   ctx_norm     : hidden_norm of the fc output (dflash.py:392) -> f16 rows
//   final_norm   : final RMSNorm (dflash.py:403) -> bf16 for the lm_head and
//                  the optional hidden-state output
//   i8_to_f16    : exact f16 copy of int8 weights (context K/V GEMM operand)
#include <algorithm>

#include "kernels.cuh"

namespace dfl {

// inv_freq_i = theta^(-2i/128) is evaluated here in fp64 and rounded to fp32
// (the same rounding as the handle's table, which the host computes once), so
// the launch reads nothing from the host and can be captured in a graph
__global__ void rope_table_kernel(int pos0, int rows, float theta, float2* __restrict__ out) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * 64) return;
  const int r = idx >> 6, i = idx & 63;
  const float inv = static_cast<float>(pow(static_cast<double>(theta), -2.0 * i / 128.0));
  const float ang = static_cast<float>(pos0 + r) * inv;
  float s, c;
  sincosf(ang, &s, &c);
  out[idx] = make_float2(c, s);
}

// map records of a forward too long to travel with rope_table_map
__global__ void kv_upload_kernel(const __grid_constant__ KvUpload up, KvSeq* __restrict__ dst) {
  griddep_wait();
  griddep_launch_dependents();
  for (int i = threadIdx.x; i < up.n; i += blockDim.x) dst[up.off + i] = up.s[i];
}

// rows of one forward: packed context rows (sequence s: positions pos0[s] + i),
// then block row m = s * block + j at pos0[s] + ctx_s + j.  With up.n > 0 the
// whole map travels in `up` (block 0 stores it at m.seq); otherwise earlier
// kv_upload launches stored it.
__global__ void rope_table_map_kernel(const __grid_constant__ KvUpload up, const KvMap m, int block,
                                      int rows, const float* __restrict__ inv_freq,
                                      float2* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < up.n; i += blockDim.x) const_cast<KvSeq*>(m.seq)[i] = up.s[i];
  const KvSeq* seq = up.n > 0 ? up.s : m.seq;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * 64) return;
  const int r = idx >> 6, i = idx & 63;
  const int nctx = seq[m.nseq].ctx_start;
  int pos;
  if (r < nctx) {
    const int s = kv_seq_of_ctx_row(seq, m.nseq, r);
    pos = seq[s].pos0 + (r - seq[s].ctx_start);
  } else {
    const int s = (r - nctx) / block, j = (r - nctx) - s * block;
    pos = seq[s].pos0 + (seq[s + 1].ctx_start - seq[s].ctx_start) + j;
  }
  const float ang = static_cast<float>(pos) * inv_freq[i];
  float sn, cs;
  sincosf(ang, &sn, &cs);
  out[idx] = make_float2(cs, sn);
}

// h = noise (fp32) with its sum of squares and max |h * w| (w: the first
// layer's input RMSNorm weight) for the limb split of the first projection;
// one CTA per row.  With `anchor` ([M / block, H], the soft anchor rows), row
// 0 of every block is read from there instead of from the noise.
__global__ void init_h_kernel(const __nv_bfloat16* __restrict__ noise, int M, int H,
                              float* __restrict__ h, float* __restrict__ hstat,
                              const float* __restrict__ w, float* __restrict__ hmax,
                              const __nv_bfloat16* __restrict__ anchor, int block) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float red[2][32];
  const int row = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const __nv_bfloat16* src = (anchor && row % block == 0) ? anchor + (size_t)(row / block) * H
                                                          : noise + (size_t)row * H;
  float ss = 0.f, mw = 0.f;
  for (int k = threadIdx.x * 8; k < H; k += blockDim.x * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + k);
    const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + k));
    const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + k + 4));
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
    float f[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 t = __bfloat1622float2(b[e]);
      f[2 * e] = t.x;
      f[2 * e + 1] = t.y;
    }
    float4* dst = reinterpret_cast<float4*>(h + (size_t)row * H + k);
    dst[0] = make_float4(f[0], f[1], f[2], f[3]);
    dst[1] = make_float4(f[4], f[5], f[6], f[7]);
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      ss += f[e] * f[e];
      mw = fmaxf(mw, fabsf(f[e] * wv[e]));
    }
  }
  ss = warp_sum(ss);
  mw = warp_max(mw);
  if (lane == 0) {
    red[0][warp] = ss;
    red[1][warp] = mw;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    float a = lane < nw ? red[0][lane] : 0.f;
    float b = lane < nw ? red[1][lane] : 0.f;
    a = warp_sum(a);
    b = warp_max(b);
    if (lane == 0) {
      hstat[row] = a;
      hmax[row] = b;
    }
  }
}

// ctx_out[r, k] = f16(raw[r, k] * rsqrt(sum_p part[p, r] / H + eps) * w[k]);
// one CTA of CN_THREADS per row.  The row's loads are issued first (up to
// CN_HELD groups of 8 values per thread stay in registers) while warp 0 sums
// the partials, so the reduction's latency hides under the row's reads.
constexpr int CN_THREADS = 128, CN_HELD = 6;
__global__ void __launch_bounds__(CN_THREADS) ctx_norm_kernel(const float* __restrict__ raw,
                                                              const float* __restrict__ part, int nparts,
                                                              int rows, int H, const float* __restrict__ w,
                                                              float eps, __half* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  const int r = blockIdx.x;
  __shared__ float rs;
  const float* src = raw + (size_t)r * H;
  __half* dst = out + (size_t)r * H;
  const int ng = H / 8;
  float4 v[CN_HELD][2];
#pragma unroll
  for (int i = 0; i < CN_HELD; ++i) {
    const int g = threadIdx.x + i * CN_THREADS;
    if (g < ng) {
      v[i][0] = *reinterpret_cast<const float4*>(src + 8 * g);
      v[i][1] = *reinterpret_cast<const float4*>(src + 8 * g + 4);
    }
  }
  if (threadIdx.x < 32) {
    float ss = 0.f;
    for (int q = threadIdx.x; q < nparts; q += 32) ss += part[(size_t)q * rows + r];
    ss = warp_sum(ss);
    if (threadIdx.x == 0) rs = rsqrtf(ss / static_cast<float>(H) + eps);
  }
  __syncthreads();
  const float rstd = rs;
  auto put = [&](int g, const float4& a, const float4& c) {
    const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + 8 * g));
    const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + 8 * g + 4));
    uint4 o;
    o.x = pack_f16x2(a.x * rstd * w0.x, a.y * rstd * w0.y);
    o.y = pack_f16x2(a.z * rstd * w0.z, a.w * rstd * w0.w);
    o.z = pack_f16x2(c.x * rstd * w1.x, c.y * rstd * w1.y);
    o.w = pack_f16x2(c.z * rstd * w1.z, c.w * rstd * w1.w);
    *reinterpret_cast<uint4*>(dst + 8 * g) = o;
  };
#pragma unroll
  for (int i = 0; i < CN_HELD; ++i) {
    const int g = threadIdx.x + i * CN_THREADS;
    if (g < ng) put(g, v[i][0], v[i][1]);
  }
  for (int g = threadIdx.x + CN_HELD * CN_THREADS; g < ng; g += CN_THREADS)   // rows wider than held
    put(g, *reinterpret_cast<const float4*>(src + 8 * g), *reinterpret_cast<const float4*>(src + 8 * g + 4));
}

// hn = bf16(h * rstd * w) for every row; also the caller's hidden output
// (bf16, or fp32 when out_f32) when given
template <bool OUT_F32>
__global__ void final_norm_kernel(const float* __restrict__ h, const float* __restrict__ hstat,
                                  int hparts, int M, int H, const float* __restrict__ w, float eps,
                                  __nv_bfloat16* __restrict__ hn, void* __restrict__ out, int block,
                                  int drop_first) {
  griddep_wait();
  griddep_launch_dependents();
  const int row = blockIdx.x;
  const int j = row % block;
  const bool keep = !drop_first || j > 0;
  const int hrow = drop_first ? (row / block) * (block - 1) + j - 1 : row;
  __shared__ float rs;
  if (threadIdx.x == 0) {
    float ss = 0.f;
    for (int q = 0; q < hparts; ++q) ss += hstat[(size_t)q * M + row];
    rs = rsqrtf(ss / static_cast<float>(H) + eps);
  }
  __syncthreads();
  const float rstd = rs;
  for (int k = threadIdx.x * 4; k < H; k += blockDim.x * 4) {
    const float4 x = *reinterpret_cast<const float4*>(h + (size_t)row * H + k);
    const float4 wv = *reinterpret_cast<const float4*>(w + k);
    const float4 y = make_float4(x.x * rstd * wv.x, x.y * rstd * wv.y, x.z * rstd * wv.z,
                                 x.w * rstd * wv.w);
    uint2 o;
    o.x = pack_bf16x2(y.x, y.y);
    o.y = pack_bf16x2(y.z, y.w);
    if (keep) *reinterpret_cast<uint2*>(hn + (size_t)hrow * H + k) = o;
    if (out) {
      if (OUT_F32)
        *reinterpret_cast<float4*>(static_cast<float*>(out) + (size_t)row * H + k) = y;
      else
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + (size_t)row * H + k) = o;
    }
  }
}

__global__ void i8_to_f16_kernel(const int8_t* __restrict__ src, size_t n, __half* __restrict__ dst) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    dst[i] = __int2half_rn(static_cast<int>(src[i]));
}

__global__ void i8_to_bf16_kernel(const int8_t* __restrict__ src, size_t n, __nv_bfloat16* __restrict__ dst) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16_rn(static_cast<float>(src[i]));   // |q| <= 127: exact in bf16
}

cudaError_t i8_to_bf16_launch(const int8_t* src, size_t n, __nv_bfloat16* dst, cudaStream_t st) {
  i8_to_bf16_kernel<<<1024, 256, 0, st>>>(src, n, dst);
  return cudaGetLastError();
}

// A bounded wait that is meant to run out: one thread waits on an mbarrier
// that nothing arrives on, for `polls` tries, then records the timeout in the
// error word the way every bounded wait of the library does, and the kernel
// returns.  Used to test failure reporting without faulting anything.
__global__ void bounded_wait_probe_kernel(uint32_t polls, int* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    bool done = false;
    for (uint32_t i = 0; i < polls && !done; ++i) done = mbar_try_wait(&bar, 0);
    if (!done) atomicExch(err, kDevMbarTimeout);
  }
}

cudaError_t bounded_wait_probe_launch(uint32_t polls, int* err, cudaStream_t st) {
  bounded_wait_probe_kernel<<<1, 32, 0, st>>>(polls, err);
  return cudaGetLastError();
}

// row r of int8 [rows, K] -> f16 row (r / grp) * period + off + r % grp of dst
__global__ void i8_to_f16_rows_kernel(const int8_t* __restrict__ src, int rows, int K, __half* __restrict__ dst,
                                      int grp, int period, int off) {
  const size_t n = (size_t)rows * K;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / K), k = (int)(i - (size_t)r * K);
    const size_t dr = (size_t)(r / grp) * period + off + r % grp;
    dst[dr * K + k] = __int2half_rn(static_cast<int>(src[i]));
  }
}

cudaError_t rope_table_launch(int pos0, int rows, float theta, float2* out, cudaStream_t st) {
  if (rows < 1) return cudaSuccess;
  DFL_TRY(max_smem_carveout(rope_table_kernel));
  rope_table_kernel<<<(rows * 64 + 255) / 256, 256, 0, st>>>(pos0, rows, theta, out);
  return cudaGetLastError();
}

cudaError_t rope_table_map_launch(const KvMap& m, const KvSeq* seq, int block, const float* inv_freq,
                                  float2* out, cudaStream_t st) {
  if (m.nseq < 1 || block < 1 || !m.seq) return cudaErrorInvalidValue;
  const int n = m.nseq + 1;
  const int rows = seq[m.nseq].ctx_start + m.nseq * block;
  KvUpload up;
  up.n = 0;
  up.off = 0;
  if (n <= kKvChunk) {
    up.n = n;
    for (int i = 0; i < n; ++i) up.s[i] = seq[i];
  } else {
    DFL_TRY(max_smem_carveout(kv_upload_kernel));
    for (int off = 0; off < n; off += kKvChunk) {
      KvUpload c;
      c.off = off;
      c.n = std::min(kKvChunk, n - off);
      for (int i = 0; i < c.n; ++i) c.s[i] = seq[off + i];
      DFL_TRY(launch_pdl(kv_upload_kernel, dim3(1), dim3(256), 0, st, c, const_cast<KvSeq*>(m.seq)));
    }
  }
  DFL_TRY(max_smem_carveout(rope_table_map_kernel));
  return launch_pdl(rope_table_map_kernel, dim3((rows * 64 + 255) / 256), dim3(256), 0, st, up, m, block,
                    rows, inv_freq, out);
}
cudaError_t init_h_launch(const __nv_bfloat16* noise, int M, int H, float* h, float* hstat,
                          const float* w, float* hmax, const __nv_bfloat16* anchor, int block,
                          cudaStream_t st) {
  if (H % 8 || block < 1) return cudaErrorInvalidValue;
  DFL_TRY(max_smem_carveout(init_h_kernel));
  return launch_pdl(init_h_kernel, dim3(M), dim3(256), 0, st, noise, M, H, h, hstat, w, hmax, anchor,
                    block);
}
cudaError_t ctx_norm_launch(const float* raw, const float* part, int nparts, int rows, int H,
                            const float* w, float eps, __half* out, cudaStream_t st) {
  if (H % 8 || rows < 1) return cudaErrorInvalidValue;
  DFL_TRY(max_smem_carveout(ctx_norm_kernel));
  return launch_pdl(ctx_norm_kernel, dim3(rows), dim3(CN_THREADS), 0, st, raw, part, nparts, rows, H, w, eps, out);
}
cudaError_t final_norm_launch(const float* h, const float* hstat, int hparts, int M, int H,
                              const float* w, float eps, __nv_bfloat16* hn, void* out, bool out_f32,
                              cudaStream_t st, int block, int drop_first) {
  if (H % 4 || block < 1 || (drop_first && (block < 2 || M % block))) return cudaErrorInvalidValue;
  const cudaError_t ce = out_f32 ? max_smem_carveout(final_norm_kernel<true>)
                                 : max_smem_carveout(final_norm_kernel<false>);
  if (ce != cudaSuccess) return ce;
  if (out_f32)
    return launch_pdl(final_norm_kernel<true>, dim3(M), dim3(256), 0, st, h, hstat, hparts, M, H, w, eps,
                      hn, out, block, drop_first);
  return launch_pdl(final_norm_kernel<false>, dim3(M), dim3(256), 0, st, h, hstat, hparts, M, H, w, eps,
                    hn, out, block, drop_first);
}
cudaError_t i8_to_f16_launch(const int8_t* src, size_t n, __half* dst, cudaStream_t st) {
  i8_to_f16_kernel<<<1024, 256, 0, st>>>(src, n, dst);
  return cudaGetLastError();
}
cudaError_t i8_to_f16_rows_launch(const int8_t* src, int rows, int K, __half* dst, int grp, int period,
                                   int off, cudaStream_t st) {
  if (rows < 1 || K < 1 || grp < 1) return cudaErrorInvalidValue;
  i8_to_f16_rows_kernel<<<2048, 256, 0, st>>>(src, rows, K, dst, grp, period, off);
  return cudaGetLastError();
}



}  // namespace dfl
