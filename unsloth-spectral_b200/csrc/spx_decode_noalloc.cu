// spx_decode_attn_noalloc: decode attention whose scratch memory is a fixed array built
// into the library, for callers that cannot allocate device memory.
//
// The array below is reserved per device for the lifetime of the process as soon as this
// file's module is loaded on that device (with CUDA's lazy module loading, the first call
// of this entry point on the device).  All calls on a device share it.
#include <mutex>

#include "spx_common.cuh"
#include "spx_decode.cuh"

namespace spx {

static __device__ __align__(256) unsigned char g_noalloc_scratch[SPX_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch array on the current device.  The first call on a device
// translates the symbol with cudaGetSymbolAddress (with that device current) and keeps
// the result; later calls only read it.
static int noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* addr[128] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  SPX_REQUIRE(e == cudaSuccess, SPX_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  SPX_REQUIRE(dev >= 0 && dev < 128, SPX_ERR_DEVICE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    SPX_REQUIRE(e == cudaSuccess && p != nullptr, SPX_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s",
                cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return SPX_OK;
}

int decode_params(const spx_decode_args* a, DecodeParams* p);

}  // namespace spx

using namespace spx;

extern "C" {

int spx_decode_attn_noalloc(const spx_decode_args* a, void* stream) {
  DecodeParams p;
  int rc = decode_params(a, &p);
  if (rc != SPX_OK) return rc;
  const size_t need = decode_workspace_bytes(p);
  SPX_REQUIRE(need <= (size_t)SPX_NOALLOC_SCRATCH_BYTES, SPX_ERR_WORKSPACE,
              "this decode needs %zu bytes of scratch; the built-in scratch holds %zu bytes "
              "(use spx_decode_attn with a caller-provided workspace)",
              need, (size_t)SPX_NOALLOC_SCRATCH_BYTES);
  void* base = nullptr;
  rc = noalloc_scratch(&base);
  if (rc != SPX_OK) return rc;
  decode_set_workspace(&p, base);
  return decode_dispatch(p, (cudaStream_t)stream);
}

}  // extern "C"
