// One-time weight preparation: the reference-exact int8 quantiser and the
// per-output-channel scale expansion into the tile order of the W8A16 kernel.
#include "kernels.cuh"

namespace dfl {

// Source channel r lands on output channel d = (r / grp) * gstride + r % grp + base
// (plain copy: grp >= n_src; gate/up interleave: grp 64, gstride 128, base 0 / 64).
__device__ __forceinline__ int w8_dst_channel(int r, int grp, int gstride, int base) {
  return (r / grp) * gstride + r % grp + base;
}

__global__ void w8_scale_kernel(const __half* __restrict__ s, int n_src, float* __restrict__ dst,
                                int grp, int gstride, int base) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n_src) return;
  dst[w8_dst_channel(r, grp, gstride, base)] = __half2float(s[r]);
}

// ------------------------------------------------------------------ quantiser
// ane_model.py:265-279: s = max|w|/127 (zero row -> 1/127), q = clip(rne(w/s))
__global__ void quantize_q8_kernel(const float* __restrict__ w, int ic, int8_t* __restrict__ q,
                                   __half* __restrict__ s) {
  const int row = blockIdx.x;
  const float* wr = w + (size_t)row * ic;
  float mx = 0.f;
  for (int k = threadIdx.x; k < ic; k += blockDim.x) mx = fmaxf(mx, fabsf(wr[k]));
  __shared__ float red[32];
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  float maxv = red[0];
  if (maxv == 0.f) maxv = 1.0f;
  const float sc = __fdiv_rn(maxv, 127.0f);
  for (int k = threadIdx.x; k < ic; k += blockDim.x) {
    float t = rintf(__fdiv_rn(wr[k], sc));
    t = fminf(fmaxf(t, -127.f), 127.f);
    q[(size_t)row * ic + k] = static_cast<int8_t>(t);
  }
  if (threadIdx.x == 0) s[row] = __float2half_rn(sc);
}

cudaError_t w8_scale_launch(const __half* s, int n_src, float* dst, int grp, int gstride,
                            int base, cudaStream_t st) {
  w8_scale_kernel<<<(n_src + 255) / 256, 256, 0, st>>>(s, n_src, dst, grp, gstride, base);
  return cudaGetLastError();
}

cudaError_t quantize_q8_launch(const float* w, int oc, int ic, int8_t* q, __half* s,
                               cudaStream_t st) {
  if (oc < 1 || ic < 1) return cudaErrorInvalidValue;
  quantize_q8_kernel<<<oc, 256, 0, st>>>(w, ic, q, s);
  return cudaGetLastError();
}

}  // namespace dfl
