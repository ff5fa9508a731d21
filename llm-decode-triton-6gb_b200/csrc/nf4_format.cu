// bitsandbytes NF4 storage-format kernels: bit-exact dequant, blockwise quantise, double quantise.
//
// Dequant reproduces the stock path the reference validates its kernel against,
// bitsandbytes.functional.dequantize_4bit (profiling/kernels/bench_nf4.py:34): each weight is the
// fp32 product code[nib] * scale rounded once to fp16/bf16, with the nested scale computed as a
// separately rounded fp32 multiply then add (nf4_gemm.py:50-51). __fmul_rn/__fadd_rn keep the
// compiler from contracting them into an FMA.
//
// Quantise/double-quantise produce the same format on the device (used to build models); their
// rounding rules are stated in include/b200decode.h and mirrored by the CPU oracle.
#include "common.cuh"

namespace b2d {
namespace {

constexpr int kDeqThreads = 256;

// One thread per 16 packed bytes = 32 weights = half of one 64-weight block.
template <typename T, bool NESTED>
__global__ void __launch_bounds__(kDeqThreads) nf4_dequant_kernel(
    const uint8_t* __restrict__ packed, int64_t ld_packed, const void* __restrict__ absmax, int64_t ld_absmax,
    const float* __restrict__ code2, const float* __restrict__ absmax2, float offset, int64_t gblk_base,
    int64_t gblk_row_stride, const float* __restrict__ code, T* __restrict__ out, int64_t ld_out, int64_t n_rows,
    int64_t k_cols) {
  __shared__ float code_s[16 * 32];  // per-lane copies: no bank conflicts on random nibbles
  __shared__ float code2_s[256];
  const int lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 16 * 32; i += kDeqThreads) code_s[i] = code[i >> 5];
  if (NESTED)
    for (int i = threadIdx.x; i < 256; i += kDeqThreads) code2_s[i] = code2[i];
  __syncthreads();
  const int64_t units_per_row = k_cols / 32;
  const int64_t units = n_rows * units_per_row;
  for (int64_t u = blockIdx.x * static_cast<int64_t>(kDeqThreads) + threadIdx.x; u < units;
       u += static_cast<int64_t>(gridDim.x) * kDeqThreads) {
    const int64_t row = u / units_per_row;
    const int64_t k0 = (u - row * units_per_row) * 32;
    const int64_t blk = k0 >> 6;
    float sc;
    if (NESTED) {
      const uint8_t q = static_cast<const uint8_t*>(absmax)[row * ld_absmax + blk];
      const int64_t gb = gblk_base + row * gblk_row_stride + blk;
      sc = __fadd_rn(__fmul_rn(code2_s[q], absmax2[gb >> 8]), offset);
    } else {
      sc = static_cast<const float*>(absmax)[row * ld_absmax + blk];
    }
    const uint4 wv = ldg_stream_u4(packed + row * ld_packed + (k0 >> 1));
    const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[16];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        const uint32_t byte = byte_of(ws[q], bb);
        const float hi = __fmul_rn(code_s[((byte >> 4) << 5) + lane], sc);
        const float lo = __fmul_rn(code_s[((byte & 15u) << 5) + lane], sc);
        o[q * 4 + bb] = static_cast<uint32_t>(Dt<T>::bits_rn(hi)) | (static_cast<uint32_t>(Dt<T>::bits_rn(lo)) << 16);
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(out + row * ld_out + k0);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
  }
}

template <typename T>
__device__ __forceinline__ float load_as_f32(const T* p, int64_t i) { return Dt<T>::to_f32(p[i]); }
template <>
__device__ __forceinline__ float load_as_f32<float>(const float* p, int64_t i) { return p[i]; }

// Index of the nearest entry of an ascending table (ties to the lower entry), from fp32
// differences exactly as the oracle computes them.
template <int NCODE>
__device__ __forceinline__ int nearest_code(float v, const float* tab) {
  int lo = 0, hi = NCODE;                 // first index with tab[i] >= v
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (tab[mid] < v) lo = mid + 1; else hi = mid;
  }
  const int h = lo;
  if (h == 0) return 0;
  if (h >= NCODE) return NCODE - 1;
  const float d_lo = __fsub_rn(v, tab[h - 1]);
  const float d_hi = __fsub_rn(tab[h], v);
  return d_hi < d_lo ? h : h - 1;
}

// One warp per 64-value block: lane l quantises elements 2l and 2l+1 and writes byte l.
template <typename T>
__global__ void __launch_bounds__(256) nf4_quantize_kernel(const T* __restrict__ w, int64_t nblocks,
                                                           const float* __restrict__ code,
                                                           uint8_t* __restrict__ packed,
                                                           float* __restrict__ absmax) {
  __shared__ float code_s[16];
  if (threadIdx.x < 16) code_s[threadIdx.x] = code[threadIdx.x];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + (threadIdx.x >> 5); b < nblocks; b += warps) {
    const float v0 = load_as_f32(w, b * 64 + 2 * lane);
    const float v1 = load_as_f32(w, b * 64 + 2 * lane + 1);
    float m = fmaxf(fabsf(v0), fabsf(v1));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float r = m > 0.f ? __frcp_rn(m) : 0.f;
    const int i0 = nearest_code<16>(__fmul_rn(v0, r), code_s);
    const int i1 = nearest_code<16>(__fmul_rn(v1, r), code_s);
    packed[b * 32 + lane] = static_cast<uint8_t>((i0 << 4) | i1);
    if (lane == 0) absmax[b] = m;
  }
}

// Fixed-order float64 mean: 1024 strided partial sums, then the partials in order.
__global__ void __launch_bounds__(1024) fixed_order_mean_kernel(const float* __restrict__ a, int64_t n,
                                                                float* __restrict__ out) {
  __shared__ double part[1024];
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += 1024) s = s + static_cast<double>(a[i]);
  part[threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < 1024; ++i) t = t + part[i];
    out[0] = __double2float_rn(t / static_cast<double>(n));
  }
}

// One 256-thread CTA per group of 256 scales.
__global__ void __launch_bounds__(256) double_quant_kernel(const float* __restrict__ absmax, int64_t n,
                                                           const float* __restrict__ code2,
                                                           const float* __restrict__ offset_p,
                                                           uint8_t* __restrict__ q, float* __restrict__ absmax2) {
  __shared__ float code2_s[256];
  __shared__ float red[8];
  code2_s[threadIdx.x] = code2[threadIdx.x];
  const float offset = *offset_p;
  const int64_t i = blockIdx.x * 256LL + threadIdx.x;
  const float a = i < n ? __fsub_rn(absmax[i], offset) : 0.f;
  float m = fabsf(a);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float gm = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) gm = fmaxf(gm, red[w]);
  const float r = gm > 0.f ? __frcp_rn(gm) : 0.f;
  if (i < n) q[i] = static_cast<uint8_t>(nearest_code<256>(__fmul_rn(a, r), code2_s));
  if (threadIdx.x == 0) absmax2[blockIdx.x] = gm;
}

int grid_for(int64_t work, int per_cta, const DeviceInfo& di) {
  int64_t g = (work + per_cta - 1) / per_cta;
  const int64_t cap = static_cast<int64_t>(di.sm_count) * 16;
  if (g > cap) g = cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace b2d

using namespace b2d;

extern "C" int b2d_nf4_dequant(const uint8_t* packed, int64_t ld_packed, const void* absmax, int64_t ld_absmax,
                               int nested, const float* code2, const float* absmax2, float offset, int64_t gblk_base,
                               int64_t gblk_row_stride, const float* code, void* out, int64_t ld_out, int64_t n_rows,
                               int64_t k_cols, int dtype, void* stream) {
  if (n_rows < 0 || k_cols < 0) return B2D_ERR_ARG;
  if (dtype != B2D_F16 && dtype != B2D_BF16) return B2D_ERR_DTYPE;
  if (k_cols % 64 != 0) return B2D_ERR_SHAPE;
  if (n_rows == 0 || k_cols == 0) return B2D_OK;
  if (!packed || !absmax || !code || !out || (nested && (!code2 || !absmax2))) return B2D_ERR_ARG;
  if (ld_packed < k_cols / 2 || ld_absmax < k_cols / 64 || ld_out < k_cols) return B2D_ERR_SHAPE;
  if (!aligned(packed, 16) || ld_packed % 16 || !aligned(out, 16) || ld_out % 8) return B2D_ERR_ALIGN;
  DeviceInfo di;
  int st = device_info(&di);
  if (st != B2D_OK) return st;
  const int grid = grid_for(n_rows * (k_cols / 32), kDeqThreads, di);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define B2D_DEQ(T, NEST)                                                                                    \
  nf4_dequant_kernel<T, NEST><<<grid, kDeqThreads, 0, s>>>(packed, ld_packed, absmax, ld_absmax, code2,     \
                                                           absmax2, offset, gblk_base, gblk_row_stride, code, \
                                                           static_cast<T*>(out), ld_out, n_rows, k_cols)
  if (dtype == B2D_F16) {
    if (nested) B2D_DEQ(__half, true); else B2D_DEQ(__half, false);
  } else {
    if (nested) B2D_DEQ(__nv_bfloat16, true); else B2D_DEQ(__nv_bfloat16, false);
  }
#undef B2D_DEQ
  return launch_status();
}

extern "C" int b2d_nf4_quantize(const void* w, int64_t n, int dtype, const float* code, uint8_t* packed,
                                float* absmax, void* stream) {
  if (n < 0) return B2D_ERR_ARG;
  if (n % 64 != 0) return B2D_ERR_SHAPE;
  if (dtype != B2D_F16 && dtype != B2D_BF16 && dtype != B2D_F32) return B2D_ERR_DTYPE;
  if (n == 0) return B2D_OK;
  if (!w || !code || !packed || !absmax) return B2D_ERR_ARG;
  DeviceInfo di;
  int st = device_info(&di);
  if (st != B2D_OK) return st;
  const int64_t nb = n / 64;
  const int grid = grid_for(nb, 8, di);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B2D_F32)
    nf4_quantize_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(w), nb, code, packed, absmax);
  else if (dtype == B2D_F16)
    nf4_quantize_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(w), nb, code, packed, absmax);
  else
    nf4_quantize_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(w), nb, code, packed,
                                                            absmax);
  return launch_status();
}

extern "C" int b2d_nf4_double_quant(const float* absmax, int64_t n_blocks, const float* code2, uint8_t* qabsmax,
                                    float* absmax2, float* offset_out, void* stream) {
  if (n_blocks < 0) return B2D_ERR_ARG;
  if (n_blocks == 0) return B2D_OK;
  if (!absmax || !code2 || !qabsmax || !absmax2 || !offset_out) return B2D_ERR_ARG;
  DeviceInfo di;
  int st = device_info(&di);
  if (st != B2D_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  fixed_order_mean_kernel<<<1, 1024, 0, s>>>(absmax, n_blocks, offset_out);
  if ((st = launch_status()) != B2D_OK) return st;
  const int64_t groups = (n_blocks + 255) / 256;
  if (groups > 0x7fffffff) return B2D_ERR_SHAPE;
  double_quant_kernel<<<static_cast<unsigned>(groups), 256, 0, s>>>(absmax, n_blocks, code2, offset_out, qabsmax,
                                                                     absmax2);
  return launch_status();
}
