// RMSNorm of the model loop's hidden rows, with the residual add fused in front of it
// (spx_rmsnorm, include/spx.h).  One CTA of 256 threads per row, the row held in
// registers (16-byte vectors, dim <= 8192), the sum of squares reduced in float32.
//   h   = x (+ residual), rounded to the row type (the residual stream keeps it)
//   out = T(h * rsqrt(mean(h^2) + eps)) * weight   (the product rounded to T)
// which is the arithmetic of the usual `(x.float() * rsqrt(x.float().pow(2).mean(-1) +
// eps)).to(T) * weight` and `h = h + a` in T, up to the summation order of the mean.
#include "spx_common.cuh"

namespace spx {
namespace nrm {

constexpr int NT = 256;
constexpr int VMAX = 4;   // 16-byte vectors per thread: dim <= 256 * 8 * 4 = 8192

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename T>
__global__ void __launch_bounds__(NT) rmsnorm_kernel(const T* x, const T* res,
                                                     const T* __restrict__ w, T* __restrict__ out,
                                                     T* hout, int dim, float eps) {
  __shared__ float red[NT / 32];
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, nv = dim / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * dim);
  const uint4* rr = res ? reinterpret_cast<const uint4*>(res + row * dim) : nullptr;
  float h[VMAX][8];
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < VMAX; ++q) {
    const int v = tid + q * NT;
    if (v < nv) {
      const uint4 a = xr[v];
      const T* ae = reinterpret_cast<const T*>(&a);
      uint4 b = make_uint4(0u, 0u, 0u, 0u);
      if (rr) b = rr[v];
      const T* be = reinterpret_cast<const T*>(&b);
      uint4 ho;
      T* he = reinterpret_cast<T*>(&ho);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const T hv = rr ? from_f<T>(to_f(ae[e]) + to_f(be[e])) : ae[e];
        he[e] = hv;
        h[q][e] = to_f(hv);
        ss = fmaf(h[q][e], h[q][e], ss);
      }
      if (rr) reinterpret_cast<uint4*>(hout + row * dim)[v] = ho;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < NT / 32; ++k) tot += red[k];
  const float inv = rsqrtf(tot / (float)dim + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
#pragma unroll
  for (int q = 0; q < VMAX; ++q) {
    const int v = tid + q * NT;
    if (v < nv) {
      const uint4 wv = wr[v];
      const T* we = reinterpret_cast<const T*>(&wv);
      uint4 o;
      T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) oe[e] = from_f<T>(to_f(from_f<T>(h[q][e] * inv)) * to_f(we[e]));
      reinterpret_cast<uint4*>(out + row * dim)[v] = o;
    }
  }
}

}  // namespace nrm
}  // namespace spx

using namespace spx;

int spx_rmsnorm(const void* x, const void* residual, const void* weight, void* out,
                                   void* residual_out, int64_t rows, int dim, float eps, int dtype, void* stream) {
  SPX_REQUIRE(x && weight && out, SPX_ERR_NULL, "spx_rmsnorm: x, weight and out are required");
  SPX_REQUIRE(!residual == !residual_out, SPX_ERR_NULL,
              "spx_rmsnorm: residual and residual_out are given together or not at all");
  SPX_REQUIRE(dtype == SPX_F16 || dtype == SPX_BF16, SPX_ERR_UNSUPPORTED, "spx_rmsnorm: dtype must be F16 or BF16");
  SPX_REQUIRE(rows >= 0 && rows <= 0x7fffffff, SPX_ERR_SHAPE, "spx_rmsnorm: rows %lld out of range", (long long)rows);
  SPX_REQUIRE(dim >= 8 && dim % 8 == 0 && dim <= nrm::NT * 8 * nrm::VMAX, SPX_ERR_SHAPE,
              "spx_rmsnorm: dim %d must be a multiple of 8 in [8, %d]", dim, nrm::NT * 8 * nrm::VMAX);
  SPX_REQUIRE(eps >= 0.f, SPX_ERR_SHAPE, "spx_rmsnorm: eps must be >= 0");
  SPX_REQUIRE(aligned16(x) && aligned16(weight) && aligned16(out) && (!residual || aligned16(residual)) &&
                  (!residual_out || aligned16(residual_out)),
              SPX_ERR_ALIGN, "spx_rmsnorm: every pointer must be 16-byte aligned");
  if (rows == 0) return SPX_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == SPX_BF16)
    nrm::rmsnorm_kernel<__nv_bfloat16><<<(unsigned)rows, nrm::NT, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(residual),
        static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(out),
        static_cast<__nv_bfloat16*>(residual_out), dim, eps);
  else
    nrm::rmsnorm_kernel<__half><<<(unsigned)rows, nrm::NT, 0, st>>>(
        static_cast<const __half*>(x), static_cast<const __half*>(residual), static_cast<const __half*>(weight),
        static_cast<__half*>(out), static_cast<__half*>(residual_out), dim, eps);
  return launch_status("rmsnorm_kernel");
}
