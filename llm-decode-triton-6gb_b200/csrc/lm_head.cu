// lm_head GEMV + greedy argmax for decode (sm_100a): logits[M, V] = x[M, K] @ W[V, K]^T in fp16/bf16 with
// fp32 accumulation, and the index of each row's largest logit, in one launch (M <= 64 tokens).
//
// The reference's decode step runs `lm_head` as a cuBLAS GEMV followed by a separate `argmax`
// (profiling/common.py decode_step: model forward -> logits[:, -1].argmax(-1)); the weight (V x K fp16,
// 262 MB for Mistral-7B) is read once per step, so the kernel is HBM-bound. Here:
//  * CTA = 8 warps on a tile of 16 vocabulary rows; the warps split K (K/8 each) and every warp
//    streams its slice of the 16 rows with 16-byte loads straight into mma.sync A fragments (the
//    reduction axis is permuted per lane, identically for W and x, so each lane's 8 weights and 8
//    activations per 32-wide chunk are contiguous), 8 chunks in flight per lane (4 from 17 tokens up);
//    each A fragment feeds one MMA per 8 tokens, so the weight is read once for any batch <= 64;
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
constexpr int kLmMaxM = 64;     // tokens per launch (eight n8 MMA tiles)
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

// NT = n8 token tiles (M <= 8 NT); UNROLL = 32-wide K chunks in flight per lane.
template <typename T, int NT, int UNROLL>
__global__ void __launch_bounds__(kLmThreads, 2) lm_head_argmax_kernel(const LmArgs a) {
  pdl_launch_dependents();
  constexpr int TOK = 8 * NT;                                      // token columns
  constexpr int RPT = kLmRows * TOK >= kLmThreads ? kLmRows * TOK / kLmThreads : 1;   // rows per thread
  constexpr int GROUPS = TOK < 32 ? kLmWarps : kLmThreads / TOK;   // partial maxima per token
  __shared__ float red[kLmWarps][kLmRows][TOK];
  __shared__ long long s_part[GROUPS][TOK];
  __shared__ int s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
  const int kw = a.K / kLmWarps;                 // this warp's K slice
  const int k0 = warp * kw + tq * 8;
  const int nchunks = kw / 32;
  const T* x = static_cast<const T*>(a.x);
  const T* xr[NT];                               // token nt*8 + g (clamped: columns >= M unused)
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int tok = nt * 8 + g;
    xr[nt] = x + static_cast<int64_t>(tok < a.M ? tok : a.M - 1) * a.ldx + k0;
  }
  long long best = LLONG_MIN;                    // threads tid < M: this CTA's best key of token tid
  bool waited = false;
  if (!a.static_w) { pdl_wait(); waited = true; }
  for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x) {
    const int r0 = tile * kLmRows + g, r1 = r0 + 8;
    const T* wa = static_cast<const T*>(a.w) + static_cast<int64_t>(r0 < a.V ? r0 : a.V - 1) * a.ldw + k0;
    const T* wb = static_cast<const T*>(a.w) + static_cast<int64_t>(r1 < a.V ? r1 : a.V - 1) * a.ldw + k0;
    float c[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) c[nt][0] = c[nt][1] = c[nt][2] = c[nt][3] = 0.f;
    for (int ch = 0; ch < nchunks; ch += UNROLL) {
      uint4 va[UNROLL], vb[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        if (ch + u < nchunks) {
          va[u] = ldg_stream_u4(wa + (ch + u) * 32);
          vb[u] = ldg_stream_u4(wb + (ch + u) * 32);
        }
      }
      if (!waited) { pdl_wait(); waited = true; }   // x is the previous kernel's output
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        if (ch + u < nchunks) {
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const uint4 vx = ld_x_u4(xr[nt] + (ch + u) * 32);   // x slice: L1-resident after the first tile
            Mma<T>::run(c[nt], va[u].x, vb[u].x, va[u].y, vb[u].y, vx.x, vx.y);
            Mma<T>::run(c[nt], va[u].z, vb[u].z, va[u].w, vb[u].w, vx.z, vx.w);
          }
        }
      }
    }
    // C fragment of token tile nt: c0, c1 = row g, tokens 8nt + 2tq, +1; c2, c3 = row g + 8
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      red[warp][g][8 * nt + 2 * tq] = c[nt][0];
      red[warp][g][8 * nt + 2 * tq + 1] = c[nt][1];
      red[warp][g + 8][8 * nt + 2 * tq] = c[nt][2];
      red[warp][g + 8][8 * nt + 2 * tq + 1] = c[nt][3];
    }
    __syncthreads();
    // thread (row group rg, token tok): RPT rows of the tile for one token; the warps' partials are added in
    // warp order and rounded once to the model dtype (the logits torch would hold), and the thread keeps
    // the largest argmax key of its rows
    {
      const int tok = tid % TOK, rg = tid / TOK;
      long long key = LLONG_MIN;
      if (rg * RPT < kLmRows) {
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          const int row = rg * RPT + i;
          float s = 0.f;
#pragma unroll
          for (int w = 0; w < kLmWarps; ++w) s += red[w][row][tok];
          const int64_t vr = static_cast<int64_t>(tile) * kLmRows + row;
          const T h = Dt<T>::from_f32(s);
          if (vr < a.V && tok < a.M) {
            if (a.logits) static_cast<T*>(a.logits)[tok * a.ldl + vr] = h;
            const long long k = argmax_key(Dt<T>::to_f32(h), a.vocab_offset + vr);
            key = k > key ? k : key;
          }
        }
      }
      // row groups sharing a warp reduce through shuffles first (lane = local row group * TOK + tok)
#pragma unroll
      for (int o = TOK; o < 32; o <<= 1) {
        const long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
      }
      if (TOK < 32) {
        if (lane < TOK) s_part[warp][tok] = key;
      } else {
        s_part[rg][tok] = key;
      }
    }
    __syncthreads();
    if (tid < TOK) {
#pragma unroll
      for (int w = 0; w < GROUPS; ++w) best = s_part[w][tid] > best ? s_part[w][tid] : best;
    }
    __syncthreads();   // red / s_part are rewritten by the next tile
  }
  if (!waited) pdl_wait();
  // publish this CTA's best keys; the last CTA merges every slot in CTA order
  if (tid < TOK) {
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

template <typename T>
int launch_lm(const LmArgs& a, int grid, cudaStream_t s, bool pdl) {
  if (a.M <= 8) return launch_kernel(lm_head_argmax_kernel<T, 1, 8>, dim3(grid), dim3(kLmThreads), 0, s, pdl, a);
  if (a.M <= 16) return launch_kernel(lm_head_argmax_kernel<T, 2, 8>, dim3(grid), dim3(kLmThreads), 0, s, pdl, a);
  if (a.M <= 32) return launch_kernel(lm_head_argmax_kernel<T, 4, 4>, dim3(grid), dim3(kLmThreads), 0, s, pdl, a);
  return launch_kernel(lm_head_argmax_kernel<T, 8, 4>, dim3(grid), dim3(kLmThreads), 0, s, pdl, a);
}

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
  if (dtype == B2D_F16) return launch_lm<__half>(a, grid, s, pdl);
  return launch_lm<__nv_bfloat16>(a, grid, s, pdl);
}
