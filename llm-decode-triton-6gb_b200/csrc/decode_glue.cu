// Decode-step glue kernels for a Mistral decoder layer (sm_100a): residual add + RMSNorm, rotary
// embedding + KV-cache append, SiLU * mul. No counterpart in the reference, whose decode step runs
// these as separate torch ops inside transformers' MistralDecoderLayer (MistralRMSNorm,
// apply_rotary_pos_emb, DynamicCache.update, act_fn(gate) * up, the residual adds); here each is one
// small kernel that can be launched as a programmatic dependent of the kernel before it, so a whole
// layer is 9 launches with no host round trip. Every intermediate is rounded to the model dtype
// exactly where the torch code rounds (each elementwise torch op on fp16/bf16 tensors computes in
// fp32 and rounds its result).
#include "common.cuh"

namespace b2d {
namespace {

template <typename T>
__device__ __forceinline__ float rnd(float v) { return Dt<T>::to_f32(Dt<T>::from_f32(v)); }

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = Dt<T>::to_f32(h[i]);
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = Dt<T>::pack2(f[2 * i], f[2 * i + 1]);
  return u;
}

// ------------------------------------------------------------------ residual add + RMSNorm
constexpr int kNormThreads = 256;
constexpr int kNormMaxChunks = 4;   // 8 elements each: D <= 256 * 8 * 4 = 8192

template <typename T>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(const T* x, int64_t ldx, T* res, int64_t ldr,
                                                                   const T* weight, float eps, T* out, int64_t ldo,
                                                                   int D) {
  pdl_launch_dependents();
  __shared__ float s_part[kNormThreads / 32];
  const int row = blockIdx.x, tid = threadIdx.x;
  const int nchunk = D / 8;
  uint4 wq[kNormMaxChunks];   // the norm weight is a model parameter: fetched before the wait
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    const int ci = tid + c * kNormThreads;
    if (ci < nchunk) wq[c] = __ldg(reinterpret_cast<const uint4*>(weight + ci * 8));
  }
  pdl_wait();
  float h[kNormMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    const int ci = tid + c * kNormThreads;
    if (ci < nchunk) {
      unpack8<T>(*reinterpret_cast<const uint4*>(res + row * ldr + ci * 8), h[c]);
      if (x) {
        float xv[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(x + row * ldx + ci * 8), xv);
#pragma unroll
        for (int i = 0; i < 8; ++i) h[c][i] = rnd<T>(h[c][i] + xv[i]);   // residual + hidden_states
        *reinterpret_cast<uint4*>(res + row * ldr + ci * 8) = pack8<T>(h[c]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(h[c][i], h[c][i], ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) s_part[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += s_part[w];
  const float rstd = rsqrtf(tot / static_cast<float>(D) + eps);
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    const int ci = tid + c * kNormThreads;
    if (ci < nchunk) {
      float wv[8], o[8];
      unpack8<T>(wq[c], wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = wv[i] * rnd<T>(h[c][i] * rstd);   // weight * hidden.to(dtype)
      *reinterpret_cast<uint4*>(out + row * ldo + ci * 8) = pack8<T>(o);
    }
  }
}

// ------------------------------------------------------------------ all-reduce consumer + add + RMSNorm
// The partials of a GEMM with the all-reduce epilogue arrive as flag-in-word words, word
// (t / 2) * D + n holding tokens t, t + 1 (t even) of column n. One CTA per token pair; thread tid
// owns the same 8-column chunks as in add_rmsnorm_kernel, and every sum is formed in the same order
// (peers in rank order; squares per thread, then warps, then the CTA), so the result has the bits of
// b2d_allreduce followed by b2d_add_rmsnorm.
// Polls a thread makes in one launch before it gives up on its peers (about a second); once a rank
// has recorded an error, later launches poll once and return, so a missing peer costs one timeout.
constexpr long long kArConsumerSpin = 1LL << 22;

template <typename T>
__global__ void __launch_bounds__(kNormThreads) allreduce_add_rmsnorm_kernel(const ArPeers a, T* res, int64_t ldr,
                                                                             const T* weight, float eps, T* out,
                                                                             int64_t ldo, int M, int D) {
  pdl_launch_dependents();
  __shared__ float s_part[2][kNormThreads / 32];
  const int tp = blockIdx.x, tid = threadIdx.x;
  const int nchunk = D / 8;
  const bool two = 2 * tp + 1 < M;
  uint4 wq[kNormMaxChunks];
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    const int ci = tid + c * kNormThreads;
    if (ci < nchunk) wq[c] = __ldg(reinterpret_cast<const uint4*>(weight + ci * 8));
  }
  pdl_wait();   // the epoch counter and the residual belong to the stream order from here on
  const uint32_t e = ar_epoch(a);
  int* errors = reinterpret_cast<int*>(a.peer[a.rank] + 256);
  long long budget = *reinterpret_cast<volatile int*>(errors) == 0 ? kArConsumerSpin : 0;
  float h[2][kNormMaxChunks][8];
  float ss[2] = {0.f, 0.f};
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    const int ci = tid + c * kNormThreads;
    if (ci < nchunk) {
      float x[2][8];
#pragma unroll
      for (int i = 0; i < 8; ++i) x[0][i] = x[1][i] = 0.f;
      for (int p = 0; p < a.world; ++p) {
        const uint64_t* q = ar_slot(a, a.rank, p, e) + static_cast<int64_t>(tp) * D + ci * 8;
        uint64_t w[8];
        for (;;) {
#pragma unroll
          for (int j = 0; j < 4; ++j) ld_word2(q + 2 * j, w[2 * j], w[2 * j + 1]);
          bool ok = true;
#pragma unroll
          for (int j = 0; j < 8; ++j) ok &= static_cast<uint32_t>(w[j] >> 32) == e;
          if (ok || budget <= 0) break;
          if (--budget == 0) {
            atomicAdd(errors, 1);
            break;
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t d = static_cast<uint32_t>(w[j]);
          const T* hv = reinterpret_cast<const T*>(&d);
          x[0][j] += Dt<T>::to_f32(hv[0]);
          x[1][j] += Dt<T>::to_f32(hv[1]);
        }
      }
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (t == 1 && !two) break;
        const int64_t row = 2 * tp + t;
        unpack8<T>(*reinterpret_cast<const uint4*>(res + row * ldr + ci * 8), h[t][c]);
#pragma unroll
        for (int i = 0; i < 8; ++i) h[t][c][i] = rnd<T>(h[t][c][i] + rnd<T>(x[t][i]));   // residual + all-reduced
        *reinterpret_cast<uint4*>(res + row * ldr + ci * 8) = pack8<T>(h[t][c]);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss[t] = fmaf(h[t][c][i], h[t][c][i], ss[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < 2; ++t) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss[t] += __shfl_xor_sync(0xffffffffu, ss[t], o);
    if ((tid & 31) == 0) s_part[t][tid >> 5] = ss[t];
  }
  __syncthreads();
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    if (t == 1 && !two) break;
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) tot += s_part[t][w];
    const float rstd = rsqrtf(tot / static_cast<float>(D) + eps);
    const int64_t row = 2 * tp + t;
#pragma unroll
    for (int c = 0; c < kNormMaxChunks; ++c) {
      const int ci = tid + c * kNormThreads;
      if (ci < nchunk) {
        float wv[8], o[8];
        unpack8<T>(wq[c], wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = wv[i] * rnd<T>(h[t][c][i] * rstd);
        *reinterpret_cast<uint4*>(out + row * ldo + ci * 8) = pack8<T>(o);
      }
    }
  }
}

// ------------------------------------------------------------------ rotary embedding + KV append
struct RopeArgs {
  const void* q; int64_t ldq;
  const void* k; int64_t ldk;
  const void* v; int64_t ldv;
  const int64_t* pos;
  const void* cos; const void* sin; int64_t ld_cs;
  void* q_out; int64_t sqo_b, sqo_h;
  void* kc; int64_t skc_b, skc_h, skc_s;
  void* vc; int64_t svc_b, svc_h, svc_s;
  int32_t* seqlens;
  int B, H, KVH, D, S_max;
};

constexpr int kRopeWarps = 4;

// One warp per (sequence, head): heads [0, H) are query heads, [H, H + KVH) the KV heads (K rotated
// into the cache, V copied). Lane l owns the pairs (i, i + D/2) for i in {2l, 2l+1} (+64 per pass),
// so q_out may alias q.
template <typename T>
__global__ void __launch_bounds__(kRopeWarps * 32) rope_kv_append_kernel(const RopeArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kRopeWarps + (threadIdx.x >> 5);
  const int heads = a.H + a.KVH;
  if (gw >= a.B * heads) return;
  const int b = gw / heads, hd = gw - b * heads;
  const int64_t p = a.pos[b];
  const bool ok = p >= 0 && p < a.S_max;
  if (hd == 0 && lane == 0 && a.seqlens) a.seqlens[b] = ok ? static_cast<int32_t>(p + 1) : 0;
  if (!ok) return;
  const int half = a.D / 2;
  const T* cs = static_cast<const T*>(a.cos) + p * a.ld_cs;
  const T* sn = static_cast<const T*>(a.sin) + p * a.ld_cs;
  const bool is_q = hd < a.H;
  const int kvh = hd - a.H;
  const T* src = is_q ? static_cast<const T*>(a.q) + b * a.ldq + static_cast<int64_t>(hd) * a.D
                      : static_cast<const T*>(a.k) + b * a.ldk + static_cast<int64_t>(kvh) * a.D;
  T* dst = is_q ? static_cast<T*>(a.q_out) + b * a.sqo_b + hd * a.sqo_h
                : static_cast<T*>(a.kc) + b * a.skc_b + kvh * a.skc_h + p * a.skc_s;
  for (int i = 2 * lane; i < half; i += 64) {
    float x1[2], x2[2], c1[2], c2[2], s1[2], s2[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      x1[e] = Dt<T>::to_f32(src[i + e]);
      x2[e] = Dt<T>::to_f32(src[i + half + e]);
      c1[e] = Dt<T>::to_f32(cs[i + e]);
      c2[e] = Dt<T>::to_f32(cs[i + half + e]);
      s1[e] = Dt<T>::to_f32(sn[i + e]);
      s2[e] = Dt<T>::to_f32(sn[i + half + e]);
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      // q*cos + rotate_half(q)*sin, rotate_half(q) = cat(-q[half:], q[:half])
      dst[i + e] = Dt<T>::from_f32(rnd<T>(x1[e] * c1[e]) + rnd<T>(-x2[e] * s1[e]));
      dst[i + half + e] = Dt<T>::from_f32(rnd<T>(x2[e] * c2[e]) + rnd<T>(x1[e] * s2[e]));
    }
  }
  if (!is_q) {
    const T* vs = static_cast<const T*>(a.v) + b * a.ldv + static_cast<int64_t>(kvh) * a.D;
    T* vd = static_cast<T*>(a.vc) + b * a.svc_b + kvh * a.svc_h + p * a.svc_s;
    for (int i = 2 * lane; i < a.D; i += 64)
      *reinterpret_cast<uint32_t*>(vd + i) = *reinterpret_cast<const uint32_t*>(vs + i);
  }
}

// ------------------------------------------------------------------ SiLU * mul
template <typename T>
__global__ void silu_mul_kernel(const T* gate, int64_t ldg, const T* up, int64_t ldu, T* out, int64_t ldo, int M,
                                int N) {
  pdl_launch_dependents();
  pdl_wait();
  const int per_row = N / 8;
  const int64_t total = static_cast<int64_t>(M) * per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = i / per_row, c = i - m * per_row;
    float gv[8], uv[8], o[8];
    unpack8<T>(*reinterpret_cast<const uint4*>(gate + m * ldg + c * 8), gv);
    unpack8<T>(*reinterpret_cast<const uint4*>(up + m * ldu + c * 8), uv);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = rnd<T>(gv[e] / (1.0f + expf(-gv[e]))) * uv[e];
    *reinterpret_cast<uint4*>(out + m * ldo + c * 8) = pack8<T>(o);
  }
}

}  // namespace
}  // namespace b2d

using namespace b2d;

extern "C" int b2d_add_rmsnorm(const void* x, int64_t ldx, void* residual, int64_t ldr, const void* weight, float eps,
                               void* out, int64_t ldo, int M, int D, int dtype, int flags, void* stream) {
  if (M < 0 || D < 0) return B2D_ERR_ARG;
  if (dtype != B2D_F16 && dtype != B2D_BF16) return B2D_ERR_DTYPE;
  if (D % 8 != 0 || D > kNormThreads * 8 * kNormMaxChunks) return B2D_ERR_SHAPE;
  if (M == 0 || D == 0) return B2D_OK;
  if (!residual || !weight || !out) return B2D_ERR_ARG;
  if (ldr < D || ldo < D || (x && ldx < D)) return B2D_ERR_SHAPE;
  if (!aligned(residual, 16) || !aligned(weight, 16) || !aligned(out, 16) || (x && !aligned(x, 16)) ||
      ldr % 8 || ldo % 8 || (x && ldx % 8))
    return B2D_ERR_ALIGN;
  DeviceInfo di;
  int st;
  if ((st = device_info(&di)) != B2D_OK) return st;
  const bool pdl = (flags & B2D_LAUNCH_PDL) != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B2D_F16)
    return launch_kernel(add_rmsnorm_kernel<__half>, dim3(M), dim3(kNormThreads), 0, s, pdl,
                         static_cast<const __half*>(x), ldx, static_cast<__half*>(residual), ldr,
                         static_cast<const __half*>(weight), eps, static_cast<__half*>(out), ldo, D);
  return launch_kernel(add_rmsnorm_kernel<__nv_bfloat16>, dim3(M), dim3(kNormThreads), 0, s, pdl,
                       static_cast<const __nv_bfloat16*>(x), ldx, static_cast<__nv_bfloat16*>(residual), ldr,
                       static_cast<const __nv_bfloat16*>(weight), eps, static_cast<__nv_bfloat16*>(out), ldo, D);
}

extern "C" int b2d_allreduce_add_rmsnorm(const b2d_allreduce_epilogue* ar, void* residual, int64_t ldr,
                                         const void* weight, float eps, void* out, int64_t ldo, int M, int D,
                                         int dtype, int flags, void* stream) {
  if (!ar || M < 0 || D < 0) return B2D_ERR_ARG;
  if (dtype != B2D_F16 && dtype != B2D_BF16) return B2D_ERR_DTYPE;
  if (!ar->peer_bufs || !ar->step || ar->world < 1 || ar->world > kArMaxWorld || ar->rank < 0 ||
      ar->rank >= ar->world || ar->sites < 1 || ar->site < 0 || ar->site >= ar->sites || ar->n_max % 8)
    return B2D_ERR_ARG;
  if (D % 8 != 0 || D > kNormThreads * 8 * kNormMaxChunks) return B2D_ERR_SHAPE;
  if (static_cast<int64_t>((M + 1) / 2) * D > ar->n_max / 2) return B2D_ERR_SHAPE;
  if (M == 0 || D == 0) return B2D_OK;
  if (!residual || !weight || !out) return B2D_ERR_ARG;
  if (ldr < D || ldo < D) return B2D_ERR_SHAPE;
  if (!aligned(residual, 16) || !aligned(weight, 16) || !aligned(out, 16) || ldr % 8 || ldo % 8)
    return B2D_ERR_ALIGN;
  ArPeers a{};
  for (int p = 0; p < ar->world; ++p) {
    if (!ar->peer_bufs[p] || !aligned(ar->peer_bufs[p], 256)) return B2D_ERR_ALIGN;
    a.peer[p] = static_cast<uint8_t*>(ar->peer_bufs[p]);
  }
  a.rank = ar->rank; a.world = ar->world; a.words = ar->n_max / 2;
  a.step = ar->step; a.site = ar->site; a.sites = ar->sites;
  DeviceInfo di;
  int st;
  if ((st = device_info(&di)) != B2D_OK) return st;
  const bool pdl = (flags & B2D_LAUNCH_PDL) != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((M + 1) / 2);
  if (dtype == B2D_F16)
    return launch_kernel(allreduce_add_rmsnorm_kernel<__half>, grid, dim3(kNormThreads), 0, s, pdl, a,
                         static_cast<__half*>(residual), ldr, static_cast<const __half*>(weight), eps,
                         static_cast<__half*>(out), ldo, M, D);
  return launch_kernel(allreduce_add_rmsnorm_kernel<__nv_bfloat16>, grid, dim3(kNormThreads), 0, s, pdl, a,
                       static_cast<__nv_bfloat16*>(residual), ldr, static_cast<const __nv_bfloat16*>(weight), eps,
                       static_cast<__nv_bfloat16*>(out), ldo, M, D);
}

extern "C" int b2d_rope_kv_append(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                                  const int64_t* pos, const void* cos, const void* sin, int64_t ld_cs, void* q_out,
                                  int64_t sqo_b, int64_t sqo_h, void* k_cache, int64_t skc_b, int64_t skc_h,
                                  int64_t skc_s, void* v_cache, int64_t svc_b, int64_t svc_h, int64_t svc_s,
                                  int32_t* seqlens, int B, int H, int KVH, int D, int S_max, int dtype, int flags,
                                  void* stream) {
  if (B < 0 || H < 0 || KVH < 0 || D < 0 || S_max < 0) return B2D_ERR_ARG;
  if (dtype != B2D_F16 && dtype != B2D_BF16) return B2D_ERR_DTYPE;
  if (D % 4 != 0 || D > 256 || KVH == 0 || H % KVH != 0) return B2D_ERR_SHAPE;
  if (B == 0) return B2D_OK;
  if (!q || !k || !v || !pos || !cos || !sin || !q_out || !k_cache || !v_cache) return B2D_ERR_ARG;
  if (ldq < static_cast<int64_t>(H) * D || ldk < static_cast<int64_t>(KVH) * D ||
      ldv < static_cast<int64_t>(KVH) * D || ld_cs < D)
    return B2D_ERR_SHAPE;
  // 4-byte accesses of element pairs
  if (!aligned(q, 4) || !aligned(k, 4) || !aligned(v, 4) || !aligned(q_out, 4) || !aligned(k_cache, 4) ||
      !aligned(v_cache, 4) || !aligned(cos, 4) || !aligned(sin, 4) ||
      (ldq | ldk | ldv | ld_cs | sqo_b | sqo_h | skc_b | skc_h | skc_s | svc_b | svc_h | svc_s) % 2)
    return B2D_ERR_ALIGN;
  DeviceInfo di;
  int st;
  if ((st = device_info(&di)) != B2D_OK) return st;
  RopeArgs a{q, ldq, k, ldk, v, ldv, pos, cos, sin, ld_cs, q_out, sqo_b, sqo_h, k_cache, skc_b, skc_h, skc_s,
             v_cache, svc_b, svc_h, svc_s, seqlens, B, H, KVH, D, S_max};
  const int64_t warps = static_cast<int64_t>(B) * (H + KVH);
  const int64_t blocks = (warps + kRopeWarps - 1) / kRopeWarps;
  if (blocks > (int64_t(1) << 31) - 1) return B2D_ERR_SHAPE;
  const bool pdl = (flags & B2D_LAUNCH_PDL) != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B2D_F16)
    return launch_kernel(rope_kv_append_kernel<__half>, dim3(static_cast<unsigned>(blocks)), dim3(kRopeWarps * 32), 0,
                         s, pdl, a);
  return launch_kernel(rope_kv_append_kernel<__nv_bfloat16>, dim3(static_cast<unsigned>(blocks)),
                       dim3(kRopeWarps * 32), 0, s, pdl, a);
}

extern "C" int b2d_silu_mul(const void* gate, int64_t ldg, const void* up, int64_t ldu, void* out, int64_t ldo, int M,
                            int N, int dtype, int flags, void* stream) {
  if (M < 0 || N < 0) return B2D_ERR_ARG;
  if (dtype != B2D_F16 && dtype != B2D_BF16) return B2D_ERR_DTYPE;
  if (N % 8 != 0) return B2D_ERR_SHAPE;
  if (M == 0 || N == 0) return B2D_OK;
  if (!gate || !up || !out) return B2D_ERR_ARG;
  if (ldg < N || ldu < N || ldo < N) return B2D_ERR_SHAPE;
  if (!aligned(gate, 16) || !aligned(up, 16) || !aligned(out, 16) || ldg % 8 || ldu % 8 || ldo % 8)
    return B2D_ERR_ALIGN;
  DeviceInfo di;
  int st;
  if ((st = device_info(&di)) != B2D_OK) return st;
  const int64_t total = static_cast<int64_t>(M) * (N / 8);
  int64_t blocks = (total + 255) / 256;
  if (blocks > di.sm_count * 8) blocks = di.sm_count * 8;
  const bool pdl = (flags & B2D_LAUNCH_PDL) != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B2D_F16)
    return launch_kernel(silu_mul_kernel<__half>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, pdl,
                         static_cast<const __half*>(gate), ldg, static_cast<const __half*>(up), ldu,
                         static_cast<__half*>(out), ldo, M, N);
  return launch_kernel(silu_mul_kernel<__nv_bfloat16>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, pdl,
                       static_cast<const __nv_bfloat16*>(gate), ldg, static_cast<const __nv_bfloat16*>(up), ldu,
                       static_cast<__nv_bfloat16*>(out), ldo, M, N);
}
