// lm_head GEMV + greedy argmax for decode (sm_100a): logits[M, V] = x[M, K] @ W[V, K]^T in fp16/bf16 with
// fp32 accumulation, and the index of each row's largest logit, in one launch.
//
// The reference's decode step runs `lm_head` as a cuBLAS GEMV followed by a separate `argmax`
// (profiling/common.py decode_step: model forward -> logits[:, -1].argmax(-1)); the weight (V x K fp16,
// 262 MB for Mistral-7B) is read once per step, so the kernel is HBM-bound. Here:
//  * CTA = 8 warps on a tile of 16 vocabulary rows; the warps split K (K/8 each) and every warp
//    streams its slice of the 16 rows with 16-byte loads straight into mma.sync A fragments (the
//    reduction axis is permuted per lane, identically for W and x, so each lane's 8 weights and 8
//    activations per 32-wide chunk are contiguous), 8 chunks in flight per lane;
//  * the 8 warps' partial sums are added in warp order in shared memory, rounded once to the model
//    dtype (the logits torch would hold), and each row's value enters a per-token argmax key
//    (ordered value << 32 | ~index): the largest value wins, ties go to the lowest index, which is
//    torch.argmax's rule;
//  * CTAs are persistent (two per SM) over the tiles; each writes its best key per token to a slot,
//    and the last CTA to finish (acquire-release counter) reduces the slots in CTA order and writes
//    the ids (the counter returns to zero for the next launch).
// `vocab_offset` shifts the indices for a vocabulary-parallel shard; `keys` exports the packed keys so
// that shards can be merged by taking the maximum over ranks.
#include <climits>

#include "common.cuh"

namespace b2d {
namespace {

constexpr int kLmWarps = 8;
constexpr int kLmThreads = kLmWarps * 32;
constexpr int kLmRows = 16;     // vocabulary rows per tile (one m16 MMA tile)
constexpr int kLmUnroll = 8;    // 32-wide K chunks in flight per lane
constexpr int kLmMaxM = 8;
constexpr size_t kLmCounterBytes = 256;

struct LmArgs {
  const void* x; int64_t ldx;
  const void* w; int64_t ldw;
  int M, V, K;
  int64_t vocab_offset;
  void* logits; int64_t ldl;
  int64_t* ids;
  long long* keys;
  long long* slots;    // [grid][kLmMaxM]
  int* counter;
  int tiles;
  int static_w;
};

// Orders floats as signed integers (negative values with their magnitude bits flipped), with torch.argmax's
// rules for the special values: -0 and +0 compare equal (both map to the key of +0, so the lower index
// wins), and every NaN is larger than any number (the first NaN wins).
__device__ __forceinline__ long long argmax_key(float v, int64_t index) {
  int32_t b = __float_as_int(v);
  if (v != v) b = 0x7FFFFFFF;
  else if (b == static_cast<int32_t>(0x80000000u)) b = 0;
  else if (b < 0) b ^= 0x7FFFFFFF;
  return (static_cast<long long>(b) << 32) | static_cast<long long>(0xFFFFFFFFu - static_cast<uint32_t>(index));
}

// Activation loads: x is the previous kernel's output, read only after the dependency wait, so the load
// is an ordinary coherent one in a volatile asm (a read-only-path __ldg may be scheduled above the wait).
__device__ __forceinline__ uint4 ld_x_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p)
               : "memory");
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kLmThreads, 2) lm_head_argmax_kernel(const LmArgs a) {
  pdl_launch_dependents();
  __shared__ float red[kLmWarps][kLmRows][kLmMaxM];
  __shared__ long long s_key[4][kLmMaxM];
  __shared__ int s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
  const int kw = a.K / kLmWarps;                 // this warp's K slice
  const int k0 = warp * kw + tq * 8;
  const int nchunks = kw / 32;
  const T* x = static_cast<const T*>(a.x);
  const T* xr = x + static_cast<int64_t>(g < a.M ? g : a.M - 1) * a.ldx + k0;   // clamped: columns >= M unused
  long long best = LLONG_MIN;                    // threads tid < M: this CTA's best key of token tid
  bool waited = false;
  if (!a.static_w) { pdl_wait(); waited = true; }
  for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x) {
    const int r0 = tile * kLmRows + g, r1 = r0 + 8;
    const T* wa = static_cast<const T*>(a.w) + static_cast<int64_t>(r0 < a.V ? r0 : a.V - 1) * a.ldw + k0;
    const T* wb = static_cast<const T*>(a.w) + static_cast<int64_t>(r1 < a.V ? r1 : a.V - 1) * a.ldw + k0;
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    for (int ch = 0; ch < nchunks; ch += kLmUnroll) {
      uint4 va[kLmUnroll], vb[kLmUnroll];
#pragma unroll
      for (int u = 0; u < kLmUnroll; ++u) {
        if (ch + u < nchunks) {
          va[u] = ldg_stream_u4(wa + (ch + u) * 32);
          vb[u] = ldg_stream_u4(wb + (ch + u) * 32);
        }
      }
      if (!waited) { pdl_wait(); waited = true; }   // x is the previous kernel's output
#pragma unroll
      for (int u = 0; u < kLmUnroll; ++u) {
        if (ch + u < nchunks) {
          const uint4 vx = ld_x_u4(xr + (ch + u) * 32);   // x slice: L1-resident after the first tile
          Mma<T>::run(c, va[u].x, vb[u].x, va[u].y, vb[u].y, vx.x, vx.y);
          Mma<T>::run(c, va[u].z, vb[u].z, va[u].w, vb[u].w, vx.z, vx.w);
        }
      }
    }
    // C fragment: c0, c1 = row g, tokens 2tq, 2tq+1; c2, c3 = row g + 8
    red[warp][g][2 * tq] = c[0];
    red[warp][g][2 * tq + 1] = c[1];
    red[warp][g + 8][2 * tq] = c[2];
    red[warp][g + 8][2 * tq + 1] = c[3];
    __syncthreads();
    if (tid < kLmRows * kLmMaxM) {
      const int row = tid >> 3, tok = tid & 7;
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kLmWarps; ++w) s += red[w][row][tok];
      const int64_t vr = static_cast<int64_t>(tile) * kLmRows + row;
      const T h = Dt<T>::from_f32(s);
      long long key = LLONG_MIN;
      if (vr < a.V && tok < a.M) {
        if (a.logits) static_cast<T*>(a.logits)[tok * a.ldl + vr] = h;
        key = argmax_key(Dt<T>::to_f32(h), a.vocab_offset + vr);
      }
      // max over the 4 rows of this warp (lanes tok, tok+8, tok+16, tok+24), then over the 4 warps
#pragma unroll
      for (int o = 8; o < 32; o <<= 1) {
        const long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
      }
      if (lane < kLmMaxM) s_key[warp][lane] = key;
    }
    __syncthreads();
    if (tid < kLmMaxM) {
#pragma unroll
      for (int w = 0; w < 4; ++w) best = s_key[w][tid] > best ? s_key[w][tid] : best;
    }
  }
  if (!waited) pdl_wait();
  // publish this CTA's best keys; the last CTA merges every slot in CTA order
  if (tid < kLmMaxM) {
    a.slots[blockIdx.x * kLmMaxM + tid] = best;
    __threadfence();
  }
  __syncthreads();
  if (tid == 0) s_last = atomic_add_acq_rel_gpu(a.counter, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid < a.M) {
    long long k = LLONG_MIN;
    for (int c = 0; c < static_cast<int>(gridDim.x); ++c) {
      const long long v = __ldcg(a.slots + c * kLmMaxM + tid);
      k = v > k ? v : k;
    }
    if (a.keys) a.keys[tid] = k;
    if (a.ids) a.ids[tid] = static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFLL));
  }
  if (tid == 0) *a.counter = 0;
}

int lm_grid(int tiles, int sm_count) { return tiles < 2 * sm_count ? tiles : 2 * sm_count; }

}  // namespace
}  // namespace b2d

using namespace b2d;

extern "C" size_t b2d_lm_head_workspace_bytes(int V) {
  if (V <= 0) return 0;
  const int64_t tiles = (static_cast<int64_t>(V) + kLmRows - 1) / kLmRows;
  return kLmCounterBytes + static_cast<size_t>(tiles) * kLmMaxM * sizeof(long long);
}

extern "C" int b2d_lm_head_argmax(const void* x, int64_t ldx, const void* w, int64_t ldw, int M, int V, int K,
                                  int64_t vocab_offset, void* logits, int64_t ld_logits, int64_t* ids,
                                  long long* keys, int dtype, int flags, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  if (M < 0 || V < 0 || K < 0 || vocab_offset < 0) return B2D_ERR_ARG;
  if (dtype != B2D_F16 && dtype != B2D_BF16) return B2D_ERR_DTYPE;
  if (M > kLmMaxM || K % (kLmWarps * 32) != 0 || vocab_offset + V > 0xFFFFFFFFLL) return B2D_ERR_SHAPE;
  if (M == 0 || V == 0) return B2D_OK;
  if (K == 0) return B2D_ERR_SHAPE;
  if (!x || !w || !workspace || (!ids && !keys && !logits)) return B2D_ERR_ARG;
  if (ldx < K || ldw < K || (logits && ld_logits < V)) return B2D_ERR_SHAPE;
  if (!aligned(x, 16) || !aligned(w, 16) || ldx % 8 || ldw % 8 || !aligned(workspace, 256)) return B2D_ERR_ALIGN;
  if (logits && !aligned(logits, 2)) return B2D_ERR_ALIGN;
  if (workspace_bytes < b2d_lm_head_workspace_bytes(V)) return B2D_ERR_WORKSPACE;
  DeviceInfo di;
  int st;
  if ((st = device_info(&di)) != B2D_OK) return st;
  LmArgs a{};
  a.x = x; a.ldx = ldx; a.w = w; a.ldw = ldw;
  a.M = M; a.V = V; a.K = K; a.vocab_offset = vocab_offset;
  a.logits = logits; a.ldl = ld_logits; a.ids = ids; a.keys = keys;
  a.counter = static_cast<int*>(workspace);
  a.slots = reinterpret_cast<long long*>(static_cast<uint8_t*>(workspace) + kLmCounterBytes);
  a.tiles = (V + kLmRows - 1) / kLmRows;
  a.static_w = (flags & B2D_STATIC_WEIGHTS) ? 1 : 0;
  const int grid = lm_grid(a.tiles, di.sm_count);
  const bool pdl = (flags & B2D_LAUNCH_PDL) != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B2D_F16) return launch_kernel(lm_head_argmax_kernel<__half>, dim3(grid), dim3(kLmThreads), 0, s, pdl, a);
  return launch_kernel(lm_head_argmax_kernel<__nv_bfloat16>, dim3(grid), dim3(kLmThreads), 0, s, pdl, a);
}
