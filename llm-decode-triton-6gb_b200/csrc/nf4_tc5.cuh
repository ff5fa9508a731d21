// Internal interface of the tcgen05 NF4 GEMM for token counts 9..64, csrc/nf4_tc5.cu. The C ABI entry
// points in nf4_gemm.cu try it first and fall back to the register-staged tensor-core kernel when a
// launch does not meet its rules (see nf4_tc5_gemm).
#pragma once

#include "common.cuh"

namespace b2d {

constexpr int kTc5MaxSeg = 4;
constexpr int kTc5NotApplicable = -1;   // nf4_tc5_gemm: shape/alignment rules not met, nothing launched

struct Nf4Tc5Segment {
  const uint8_t* packed;
  int64_t ld_packed;        // bytes
  const void* absmax;       // uint8 (nested) or fp32
  int64_t ld_absmax;        // elements
  const float* absmax2;
  float offset;
  int64_t gblk_base, gblk_row_stride;
  int N;
  void* y;
  int64_t ldy;
};

struct Nf4Tc5Launch {
  const void* x;
  int64_t ldx;
  int M, K;
  int dtype, y_dtype;
  int nested;
  int nseg;
  Nf4Tc5Segment seg[kTc5MaxSeg];
  const float* code_dev;    // 16 codebook values on the device
  const float* code2;       // double-quant table shared by the segments (nested)
  bool pdl;
  int* err;                 // device word counting timed-out pipeline waits (never expected to move)
};

// Launches the tcgen05 kernel, or returns kTc5NotApplicable (nothing launched) when M is outside 9..64,
// K is not a multiple of 256, a row count is not a multiple of 8, the segments do not share one code2
// table, or an alignment rule of the tensor copies or the scale loads is not met.
int nf4_tc5_gemm(const Nf4Tc5Launch& L, cudaStream_t stream);

}  // namespace b2d
