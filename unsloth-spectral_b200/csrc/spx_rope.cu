// Query RoPE of the single-token decode forward (spx_rope_rows, include/spx.h): the
// rotation that the patched forward applies to the new token's query at its position
// before calling the decode kernel, in one launch.  Half-split convention with the
// first half of the tables for both halves, each product and sum rounded in float32 as
// the float32 tensor expression rounds them:
//   out[i]     = x[i] c - x[i + h] s,   out[i + h] = x[i + h] c + x[i] s,   c, s = row pos, col i
#include "spx_common.cuh"

namespace spx {
namespace rope {

template <typename T>
__device__ __forceinline__ float ld(const T* p);
template <>
__device__ __forceinline__ float ld<__half>(const __half* p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <>
__device__ __forceinline__ float ld<float>(const float* p) { return *p; }
template <typename T>
__device__ __forceinline__ void st(T* p, float v);
template <>
__device__ __forceinline__ void st<__half>(__half* p, float v) { *p = __float2half_rn(v); }
template <>
__device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ void st<float>(float* p, float v) { *p = v; }

// grid (rows, heads), block head_dim / 2 threads
template <typename T>
__global__ void rope_rows_kernel(const T* x, int64_t x_row_stride, const float* __restrict__ cosT,
                                 const float* __restrict__ sinT, int rope_len, const int64_t* __restrict__ posd,
                                 int64_t pos_stride, int64_t pos_host, T* __restrict__ out, int heads, int hd) {
  const int row = blockIdx.x, head = blockIdx.y, i = threadIdx.x, h = hd / 2;
  int64_t pos = posd ? posd[(int64_t)row * pos_stride] : pos_host;
  pos = pos < 0 ? 0 : (pos >= rope_len ? rope_len - 1 : pos);
  const T* xr = x + (int64_t)row * x_row_stride + (int64_t)head * hd;
  const float x1 = ld(xr + i), x2 = ld(xr + i + h);
  const float c = cosT[pos * hd + i], s = sinT[pos * hd + i];
  T* o = out + ((int64_t)row * heads + head) * hd;
  st(o + i, __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
  st(o + i + h, __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
}

}  // namespace rope
}  // namespace spx

using namespace spx;

int spx_rope_rows(const void* x, int64_t x_row_stride, const float* cos_table, const float* sin_table,
                  int rope_len, const int64_t* pos_device, int64_t pos_stride, int64_t pos_host, void* out,
                  int rows, int heads, int head_dim, int dtype, void* stream) {
  SPX_REQUIRE(x && cos_table && sin_table && out, SPX_ERR_NULL, "spx_rope_rows: x, tables and out are required");
  SPX_REQUIRE(dtype_ok(dtype), SPX_ERR_UNSUPPORTED, "spx_rope_rows: bad dtype %d", dtype);
  SPX_REQUIRE(rows >= 0 && heads >= 1 && head_dim >= 2 && head_dim % 2 == 0 && head_dim <= 1024 && rope_len >= 1,
              SPX_ERR_SHAPE, "spx_rope_rows: bad shape rows %d heads %d head_dim %d rope_len %d", rows, heads,
              head_dim, rope_len);
  SPX_REQUIRE(x_row_stride >= (int64_t)heads * head_dim && pos_stride >= 0, SPX_ERR_SHAPE,
              "spx_rope_rows: row stride %lld shorter than a row", (long long)x_row_stride);
  SPX_REQUIRE(rows <= 65535 * 1024 && heads <= 65535, SPX_ERR_SHAPE, "spx_rope_rows: too many rows or heads");
  if (rows == 0) return SPX_OK;
  const dim3 grid((unsigned)rows, (unsigned)heads);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == SPX_BF16)
    rope::rope_rows_kernel<__nv_bfloat16><<<grid, head_dim / 2, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), x_row_stride, cos_table, sin_table, rope_len, pos_device, pos_stride,
        pos_host, static_cast<__nv_bfloat16*>(out), heads, head_dim);
  else if (dtype == SPX_F16)
    rope::rope_rows_kernel<__half><<<grid, head_dim / 2, 0, st>>>(
        static_cast<const __half*>(x), x_row_stride, cos_table, sin_table, rope_len, pos_device, pos_stride, pos_host,
        static_cast<__half*>(out), heads, head_dim);
  else
    rope::rope_rows_kernel<float><<<grid, head_dim / 2, 0, st>>>(
        static_cast<const float*>(x), x_row_stride, cos_table, sin_table, rope_len, pos_device, pos_stride, pos_host,
        static_cast<float*>(out), heads, head_dim);
  return launch_status("rope_rows_kernel");
}

// ---------------------------------------------------------------------------------
// One decode token appended to the hot tier at its device length (spx_hot_append): the
// key and value rows of every (sequence, head) written at hot_len, the position at
// hot_pos[hot_len], then hot_len + 1, in one CTA (every thread reads the length before
// thread 0 advances it).  A length at or past the capacity writes nothing.
namespace spx {
namespace rope {

template <typename T>
__global__ void __launch_bounds__(512) hot_append_kernel(const T* __restrict__ k, const T* __restrict__ v,
                                                         int64_t ksb, int64_t ksh, int64_t vsb, int64_t vsh,
                                                         T* __restrict__ hk, T* __restrict__ hv,
                                                         int64_t* __restrict__ hpos, int32_t* hlen,
                                                         const int64_t* __restrict__ pos, int B, int H, int D,
                                                         int cap) {
  const int len = *hlen;
  const bool room = len >= 0 && len < cap;
  const int64_t n = (int64_t)B * H * D;
  for (int64_t e = threadIdx.x; room && e < n; e += blockDim.x) {
    const int d = (int)(e % D);
    const int64_t bh = e / D;
    const int h = (int)(bh % H), b = (int)(bh / H);
    const int64_t dst = (bh * cap + len) * D + d;
    hk[dst] = k[b * ksb + h * ksh + d];
    hv[dst] = v[b * vsb + h * vsh + d];
  }
  __syncthreads();
  if (threadIdx.x == 0 && room) {
    hpos[len] = *pos;
    *hlen = len + 1;
  }
}

}  // namespace rope
}  // namespace spx

int spx_hot_append(const void* k, const void* v, int64_t k_stride_b, int64_t k_stride_h, int64_t v_stride_b,
                   int64_t v_stride_h, void* hot_k, void* hot_v, int64_t* hot_pos, int32_t* hot_len,
                   const int64_t* pos, int batch, int heads, int head_dim, int capacity, int dtype, void* stream) {
  SPX_REQUIRE(k && v && hot_k && hot_v && hot_pos && hot_len && pos, SPX_ERR_NULL,
              "spx_hot_append: every pointer is required");
  SPX_REQUIRE(dtype_ok(dtype), SPX_ERR_UNSUPPORTED, "spx_hot_append: bad dtype %d", dtype);
  SPX_REQUIRE(batch >= 1 && heads >= 1 && head_dim >= 1 && capacity >= 1, SPX_ERR_SHAPE,
              "spx_hot_append: bad shape batch %d heads %d head_dim %d capacity %d", batch, heads, head_dim,
              capacity);
  SPX_REQUIRE(k_stride_b >= 0 && k_stride_h >= 0 && v_stride_b >= 0 && v_stride_h >= 0, SPX_ERR_SHAPE,
              "spx_hot_append: negative stride");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == SPX_BF16)
    rope::hot_append_kernel<__nv_bfloat16><<<1, 512, 0, st>>>(
        static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v), k_stride_b, k_stride_h,
        v_stride_b, v_stride_h, static_cast<__nv_bfloat16*>(hot_k), static_cast<__nv_bfloat16*>(hot_v), hot_pos,
        hot_len, pos, batch, heads, head_dim, capacity);
  else if (dtype == SPX_F16)
    rope::hot_append_kernel<__half><<<1, 512, 0, st>>>(
        static_cast<const __half*>(k), static_cast<const __half*>(v), k_stride_b, k_stride_h, v_stride_b, v_stride_h,
        static_cast<__half*>(hot_k), static_cast<__half*>(hot_v), hot_pos, hot_len, pos, batch, heads, head_dim,
        capacity);
  else
    rope::hot_append_kernel<float><<<1, 512, 0, st>>>(
        static_cast<const float*>(k), static_cast<const float*>(v), k_stride_b, k_stride_h, v_stride_b, v_stride_h,
        static_cast<float*>(hot_k), static_cast<float*>(hot_v), hot_pos, hot_len, pos, batch, heads, head_dim,
        capacity);
  return launch_status("hot_append_kernel");
}
