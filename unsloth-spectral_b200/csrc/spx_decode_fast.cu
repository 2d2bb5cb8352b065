// Fast cold-tier decode path (placeholder until the tensor-core kernel lands).
#include "spx_common.cuh"
#include "spx_decode.cuh"

namespace spx {

bool decode_fast_supported(const DecodeParams&) { return false; }

int decode_fast_launch(const DecodeParams& p, cudaStream_t st) { return decode_generic(p, st); }

}  // namespace spx
