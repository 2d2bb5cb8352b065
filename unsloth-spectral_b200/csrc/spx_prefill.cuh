// Parameters of the prefill (multi-query) attention kernels (spx_prefill.cu: mma.sync
// flash attention; spx_prefill_tc.cu: tcgen05 with TMEM accumulators).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace spx {

struct PrefillParams {
  int B, Hq, H, nrep, QT, qlen, T, nblk, nbc, RK, RV, hot, HC, causal, mask_f32, rope_len;
  float scale;
  const void* q;
  const int64_t* qpos;
  const int8_t* ck;
  const int8_t* cv;
  const float* sk;
  const float* sv;
  const void* bk;
  const void* bv;
  const int64_t* bpos;
  const void* hk;
  const void* hv;
  const int64_t* hpos;
  const float* cosT;
  const float* sinT;
  const void* mask;
  int64_t msb, msh, msq;
  void* out;
};

// tcgen05 kernel (spx_prefill_tc.cu): 128-token key tiles, so blocks of a multiple of 128.
bool prefill_tc_supported(int block_size, int num_blocks);
int prefill_tc_launch(const PrefillParams& p, int dtype, cudaStream_t st);

}  // namespace spx
