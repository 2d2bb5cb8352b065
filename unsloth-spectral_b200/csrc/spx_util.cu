// Utilities, INT8 quantiser, cold-tier reconstruction and the per-block score/value
// helpers of the spx C ABI.
#include <math.h>
#include <string.h>

#include "spx_common.cuh"

namespace spx {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

// --------------------------------------------------------------------------------
// Per-group symmetric INT8 quantisation (spectral_cache.py:481-516).
// One CTA per group: min / max / abs-max reductions, then code = rint(x / scale)
// with an IEEE round-to-nearest division, exactly as the reference's float32 torch ops.
// --------------------------------------------------------------------------------
__global__ void quantize_kernel(const float* __restrict__ x, int64_t n, int8_t* __restrict__ codes,
                                float* __restrict__ scale_out, float* __restrict__ minmax,
                                float* __restrict__ dequant) {
  const int64_t g = blockIdx.x;
  const float* xg = x + g * n;
  float mn = INFINITY, mx = -INFINITY, am = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    float v = xg[i];
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
    am = fmaxf(am, fabsf(v));
  }
  __shared__ float red[3][32];
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (l == 0) {
    red[0][w] = mn;
    red[1][w] = mx;
    red[2][w] = am;
  }
  __syncthreads();
  if (w == 0) {
    mn = l < nw ? red[0][l] : INFINITY;
    mx = l < nw ? red[1][l] : -INFINITY;
    am = l < nw ? red[2][l] : 0.f;
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    }
    if (l == 0) {
      red[0][0] = mn;
      red[1][0] = mx;
      red[2][0] = __fdiv_rn(fmaxf(am, 1e-8f), 127.0f);
    }
  }
  __syncthreads();
  const float s = red[2][0];
  if (threadIdx.x == 0) {
    scale_out[g] = s;
    if (minmax) {
      minmax[2 * g] = red[0][0];
      minmax[2 * g + 1] = red[1][0];
    }
  }
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    float c = rintf(__fdiv_rn(xg[i], s));
    codes[g * n + i] = (int8_t)(int)c;
    if (dequant) dequant[g * n + i] = __fmul_rn(c, s);
  }
}

// --------------------------------------------------------------------------------
// Cold-tier reconstruction: out[b,h,j*T+t,:] = scale * codes[t,:] @ basis (get_kv).
// --------------------------------------------------------------------------------
template <typename T>
__global__ void reconstruct_kernel(spx_reconstruct_args a) {
  const int j = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int D = a.head_dim, Tb = a.block_size, R = a.rank;
  extern __shared__ float sm_basis[];  // [R][D]
  const int64_t slot = ((int64_t)b * a.num_kv_heads + h) * a.block_capacity + j;
  const T* basis = reinterpret_cast<const T*>(a.basis) + slot * R * D;
  for (int i = threadIdx.x; i < R * D; i += blockDim.x) sm_basis[i] = to_f(basis[i]);
  __syncthreads();
  const float sc = a.scale[slot];
  const int8_t* codes = a.codes + slot * (int64_t)Tb * R;
  T* out = reinterpret_cast<T*>(a.out) + (((int64_t)b * a.num_kv_heads + h) * a.out_tokens + (int64_t)j * Tb) * D;
  for (int e = threadIdx.x; e < Tb * D; e += blockDim.x) {
    const int t = e / D, d = e - t * D;
    float acc = 0.f;
    for (int r = 0; r < R; ++r) {
      const int8_t c = a.rank_major ? codes[vtile_offset(r, t, R)] : codes[(int64_t)t * R + r];
      acc = fmaf((float)c, sm_basis[r * D + d], acc);
    }
    out[(int64_t)t * D + d] = from_f<T>(acc * sc);
  }
}

// --------------------------------------------------------------------------------
// One block's scores with float coefficients, absolute-position RoPE as in
// kernels/spectral_attention.py:375-453:  score = Q . RoPE_a(K~) with K~ = C[t] @ B.
// --------------------------------------------------------------------------------
__global__ void block_scores_kernel(spx_block_score_args a) {
  const int hq = blockIdx.y, b = blockIdx.z;
  const int D = a.head_dim, half = D / 2, R = a.rank, Tb = a.block_size;
  const int g = hq / (a.num_q_heads / a.num_kv_heads);
  extern __shared__ float sm[];  // basis [R][D] then q [D]
  float* sb = sm;
  float* sq = sm + R * D;
  for (int i = threadIdx.x; i < R * D; i += blockDim.x) sb[i] = a.basis[(int64_t)g * R * D + i];
  for (int i = threadIdx.x; i < D; i += blockDim.x) sq[i] = a.q[((int64_t)b * a.num_q_heads + hq) * D + i];
  __syncthreads();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= Tb) return;
  int64_t pos = a.start_position + t;
  pos = pos < 0 ? 0 : (pos >= a.rope_len ? a.rope_len - 1 : pos);
  const float* cr = a.cos_table + pos * D;
  const float* sr = a.sin_table + pos * D;
  const float* crow = a.coeffs + ((int64_t)g * Tb + t) * R;
  float s = 0.f;
  for (int i = 0; i < half; ++i) {
    float k1 = 0.f, k2 = 0.f;
    for (int r = 0; r < R; ++r) {
      const float c = crow[r];
      k1 = fmaf(c, sb[r * D + i], k1);
      k2 = fmaf(c, sb[r * D + i + half], k2);
    }
    const float c1 = cr[i], c2 = cr[i + half], s1 = sr[i], s2 = sr[i + half];
    s = fmaf(sq[i], c1 * k1 - s2 * k2, s);
    s = fmaf(sq[i + half], s1 * k1 + c2 * k2, s);
  }
  a.scores[((int64_t)b * a.num_q_heads + hq) * Tb + t] = s;
}

// One block's values: out = (attn @ C) @ B  (kernels/spectral_attention.py:544-601).
__global__ void block_values_kernel(spx_block_value_args a) {
  const int hq = blockIdx.x, b = blockIdx.y;
  const int D = a.head_dim, R = a.rank, Tb = a.block_size;
  const int g = hq / (a.num_q_heads / a.num_kv_heads);
  extern __shared__ float vlat[];  // [R]
  const float* at = a.attn + ((int64_t)b * a.num_q_heads + hq) * Tb;
  const float* C = a.coeffs + (int64_t)g * Tb * R;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int r = w; r < R; r += nw) {
    float acc = 0.f;
    for (int t = l; t < Tb; t += 32) acc = fmaf(at[t], C[(int64_t)t * R + r], acc);
    acc = warp_sum(acc);
    if (l == 0) vlat[r] = acc;
  }
  __syncthreads();
  const float* Bm = a.basis + (int64_t)g * R * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < R; ++r) acc = fmaf(vlat[r], Bm[(int64_t)r * D + d], acc);
    a.out[((int64_t)b * a.num_q_heads + hq) * D + d] = acc;
  }
}

}  // namespace spx

using namespace spx;

extern "C" {

int spx_abi_version(void) { return SPX_ABI_VERSION; }

const char* spx_status_string(int s) {
  switch (s) {
    case SPX_OK: return "ok";
    case SPX_ERR_NULL: return "null pointer argument";
    case SPX_ERR_SHAPE: return "invalid shape argument";
    case SPX_ERR_UNSUPPORTED: return "unsupported configuration";
    case SPX_ERR_ALIGN: return "misaligned pointer";
    case SPX_ERR_WORKSPACE: return "workspace missing or too small";
    case SPX_ERR_EMPTY: return "Empty cache - no keys available";
    case SPX_ERR_CUDA: return "CUDA runtime error";
    case SPX_ERR_DEVICE: return "current device is not sm_100 (B200)";
    default: return "unknown status";
  }
}

const char* spx_last_error(void) { return g_err; }

int spx_check_device(void) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("cudaGetDevice: %s", cudaGetErrorString(e));
    return SPX_ERR_DEVICE;
  }
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) {
    set_error("device %d is sm_%d%d; this library is built for sm_100a", dev, major, minor);
    return SPX_ERR_DEVICE;
  }
  return SPX_OK;
}

int spx_quantize_int8(const spx_quant_args* a, void* stream) {
  SPX_REQUIRE(a, SPX_ERR_NULL, "args is NULL");
  SPX_REQUIRE(a->x && a->codes && a->scale, SPX_ERR_NULL, "x, codes and scale are required");
  SPX_REQUIRE(a->num_groups >= 0 && a->group_elems > 0, SPX_ERR_SHAPE, "bad quantisation shape");
  if (a->num_groups == 0) return SPX_OK;
  quantize_kernel<<<a->num_groups, 256, 0, (cudaStream_t)stream>>>(a->x, a->group_elems, a->codes, a->scale,
                                                                  a->minmax, a->dequant);
  return launch_status("quantize_kernel");
}

int spx_reconstruct(const spx_reconstruct_args* a, void* stream) {
  SPX_REQUIRE(a, SPX_ERR_NULL, "args is NULL");
  SPX_REQUIRE(a->codes && a->scale && a->basis && a->out, SPX_ERR_NULL, "null tensor");
  SPX_REQUIRE(dtype_ok(a->dtype), SPX_ERR_UNSUPPORTED, "bad dtype");
  SPX_REQUIRE(a->head_dim > 0 && a->head_dim <= 256 && a->rank > 0 && a->rank <= 64 && a->block_size > 0 &&
                  a->num_blocks >= 0 && a->num_blocks <= a->block_capacity && a->batch > 0 && a->num_kv_heads > 0 &&
                  a->out_tokens >= a->num_blocks * a->block_size,
              SPX_ERR_SHAPE, "bad reconstruct shape");
  SPX_REQUIRE(!a->rank_major || (a->rank % 8 == 0 && a->block_size % 16 == 0), SPX_ERR_SHAPE,
              "value-tile codes need rank %% 8 == 0 and block_size %% 16 == 0");
  if (a->num_blocks == 0) return SPX_OK;
  dim3 grid(a->num_blocks, a->num_kv_heads, a->batch);
  const size_t smem = (size_t)a->rank * a->head_dim * sizeof(float);
  return SPX_DISPATCH_DTYPE(a->dtype, T, [&] {
    cudaFuncSetAttribute(reconstruct_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    reconstruct_kernel<T><<<grid, 256, smem, (cudaStream_t)stream>>>(*a);
    return launch_status("reconstruct_kernel");
  });
}

int spx_block_scores(const spx_block_score_args* a, void* stream) {
  SPX_REQUIRE(a, SPX_ERR_NULL, "args is NULL");
  SPX_REQUIRE(a->q && a->coeffs && a->basis && a->cos_table && a->sin_table && a->scores, SPX_ERR_NULL,
              "null tensor");
  SPX_REQUIRE(a->head_dim > 0 && a->head_dim % 2 == 0 && a->head_dim <= 256 && a->rank > 0 && a->rank <= 128 &&
                  a->num_kv_heads > 0 && a->num_q_heads % a->num_kv_heads == 0 && a->block_size > 0 &&
                  a->batch > 0 && a->rope_len > 0,
              SPX_ERR_SHAPE, "bad block-score shape");
  const size_t smem = ((size_t)a->rank * a->head_dim + a->head_dim) * sizeof(float);
  cudaFuncSetAttribute(block_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((a->block_size + 127) / 128, a->num_q_heads, a->batch);
  block_scores_kernel<<<grid, 128, smem, (cudaStream_t)stream>>>(*a);
  return launch_status("block_scores_kernel");
}

int spx_block_values(const spx_block_value_args* a, void* stream) {
  SPX_REQUIRE(a, SPX_ERR_NULL, "args is NULL");
  SPX_REQUIRE(a->attn && a->coeffs && a->basis && a->out, SPX_ERR_NULL, "null tensor");
  SPX_REQUIRE(a->head_dim > 0 && a->rank > 0 && a->rank <= 1024 && a->num_kv_heads > 0 &&
                  a->num_q_heads % a->num_kv_heads == 0 && a->block_size > 0 && a->batch > 0,
              SPX_ERR_SHAPE, "bad block-value shape");
  dim3 grid(a->num_q_heads, a->batch);
  block_values_kernel<<<grid, 128, a->rank * sizeof(float), (cudaStream_t)stream>>>(*a);
  return launch_status("block_values_kernel");
}

}  // extern "C"
