// Internal interface of the TMA-staged NF4 GEMM for decode batches (M <= 8), csrc/nf4_gemm_tma.cu.
// The C ABI entry points in nf4_gemm.cu try it first and fall back to the register-staged kernels
// when a launch does not meet its rules (see nf4_tma_gemm).
#pragma once

#include "common.cuh"

namespace b2d {

constexpr int kTmaMaxSeg = 4;
constexpr int kTmaNotApplicable = -1;   // nf4_tma_gemm: shape/alignment rules not met, nothing launched

enum TmaMode { kTmaIndependent = 0, kTmaSiluMul = 1, kTmaAllReduce = 2 };

struct Nf4TmaSegment {
  const uint8_t* packed;
  int64_t ld_packed;        // bytes
  const void* absmax;       // uint8 (nested) or fp32
  int64_t ld_absmax;        // elements
  const float* code2;
  const float* absmax2;
  float offset;
  int64_t gblk_base, gblk_row_stride;
  int N;
  void* y;                  // independent mode: this segment's output; silu_mul: segment 0's y is the output
  int64_t ldy;
};

struct Nf4TmaLaunch {
  const void* x;
  int64_t ldx;
  int M, K;
  int dtype, y_dtype;
  int nested;
  int mode;                 // TmaMode
  int nseg;
  Nf4TmaSegment seg[kTmaMaxSeg];
  const float* code_dev;    // 16 codebook values on the device (used when code_host is null)
  const float* code_host;   // 16 codebook values on the host, passed by value
  bool pdl, static_w;
  ArPeers ar;               // kTmaAllReduce
  int* err;                 // device word counting timed-out pipeline waits (never expected to move)
};

// Launches the TMA-staged kernel, or returns kTmaNotApplicable (nothing launched) when M > 8, a row
// count is not a multiple of 8, the scale tables or their strides are not 4-byte aligned, the segments
// do not share one code2 table, or no cluster configuration keeps each warp's K slice in registers.
int nf4_tma_gemm(const Nf4TmaLaunch& L, cudaStream_t stream);

}  // namespace b2d
