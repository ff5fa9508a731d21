// Split-K flash-decoding grouped-query attention for sm_100a (one query token per sequence).
//
// Replaces the reference's _partial_kernel / _merge_kernel / decode_attention
// (profiling/kernels/decode_attention.py:18-91): every CTA owns one (sequence, KV head, key split)
// and serves all G = H/KVH query heads of that KV head, so each K/V row is read from HBM once; a
// second kernel merges the splits with a log-sum-exp combine. Adds per-sequence lengths.
//
// Partial kernel, per warp and 16-key tile (m16n8k16, fp32 accumulate):
//   S = Q K^T   A = Q (16 rows = query heads of the group, rows >= G are zero), B = K^T.
//               Thread (g,t) loads key rows g and 8+g of the tile, head-dim slice [D/4*t, D/4*t+D/4)
//               with 16-byte loads; the MMA reduction axis is permuted to match (k-step j uses
//               d = D/4*t + 4j + {0..3}), and Q is loaded in the same permuted order.
//   P = exp2(S*scale*log2e - m)   online softmax per head, max over the tile's 16 keys by a
//               quad shuffle; the S accumulator layout is the A-operand layout of the next MMA.
//   O += P V    B = V: thread (g,t) loads value rows 2t, 2t+1, 8+2t, 9+2t over the head-dim slice
//               [D/8*g, D/8*g+D/8) and pairs rows with byte permutes; output column n of n8 tile j
//               is d = D/8*(column) + j, so each thread ends up owning O[head][D/4*t .. D/4*t+D/4).
//   No shared-memory staging for K/V: 16-byte global loads straight into fragment registers, one
//   tile prefetched ahead. Warps of a CTA take interleaved tiles and merge through shared memory.
// Workspace per (b, h, split): unnormalised O[D] (fp32) and (m, l) with m in the log2 domain.
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include <atomic>
#include <mutex>

#include "common.cuh"

namespace b2d {
namespace {

constexpr int kAttnWarps = 4;
constexpr float kLog2e = 1.4426950408889634f;
// Workspace layout: a fixed-size region of per-(sequence, KV head) arrival counters first (so calls
// of any shape agree on where they live and always find them zero), then the split partials.
constexpr size_t kAttnCounterBytes = 64 * 1024;
constexpr int kMaxAttnCounters = static_cast<int>(kAttnCounterBytes / 4);
constexpr int kMaxFusedSplits = 64;   // the in-kernel combine loops over the splits per element

constexpr int kMaxL2Prefetch = 4;

struct AttnArgs {
  const void* q; int64_t sq_b, sq_h;
  const void* k; int64_t sk_b, sk_h, sk_s;
  const void* v; int64_t sv_b, sv_h, sv_s;
  const int32_t* seqlens;
  int B, H, KVH, S, G;
  float scale_log2;
  int nsplit, chunk;
  float* acc;   // [B*H*nsplit][D]
  float* ml;    // [B*H*nsplit][2]
  void* out; int64_t so_b, so_h;
  int* counters;   // [B*KVH], zero between launches
  int fused;       // 1: the last split CTA of each (b, kvh) combines and writes out
  int out_f32;     // fused: out is fp32 (else the input dtype)
  int kv_prefix;   // 1: keys before each sequence's newest one may be read before the dependency wait
  // append mode (b2d_gqa_decode_append): q holds the projection output before RoPE; the kernel rotates it,
  // rotates and appends this step's key/value at position pos[b], and writes seqlens[b] = pos[b] + 1
  int append;
  const void* k_new; int64_t ldk_new;
  const void* v_new; int64_t ldv_new;
  const int64_t* pos;
  const void* rcos; const void* rsin; int64_t ld_cs;
  int32_t* seqlens_out;
  // L2 prefetch of static data the following launches read (the next GEMMs' weights): the CTAs issue
  // bulk L2 prefetches of equal slices of each range before any dependency wait; no result depends on it
  int npf;
  const char* pf_base[kMaxL2Prefetch];
  int64_t pf_bytes[kMaxL2Prefetch];   // multiples of 16
};

template <typename T>
__device__ __forceinline__ void store_out(const AttnArgs& a, int b, int h, int d, float v) {
  if (a.out_f32) static_cast<float*>(a.out)[b * a.so_b + h * a.so_h + d] = v;
  else static_cast<T*>(a.out)[b * a.so_b + h * a.so_h + d] = Dt<T>::from_f32(v);
}

__device__ __forceinline__ int seqlen_of(const AttnArgs& a, int b) {
  if (!a.seqlens) return a.S;
  int n = a.seqlens[b];
  return n < 0 ? 0 : (n > a.S ? a.S : n);
}

template <typename T, int D>
struct KvTile {
  uint4 k[2][D / 32];   // key rows g, 8+g; head-dim slice D/4 wide
  uint4 v[4][D / 64];   // value rows 2t, 2t+1, 8+2t, 9+2t; head-dim slice D/8 wide
};

template <typename T, int D>
__device__ __forceinline__ void load_tile(KvTile<T, D>& kt, const T* kbase, const T* vbase, int64_t sk_s,
                                          int64_t sv_s, int tok0, int tend, int g, int tq) {
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int tok = tok0 + r * 8 + g;
    const T* p = kbase + static_cast<int64_t>(tok) * sk_s + (D / 4) * tq;
#pragma unroll
    for (int i = 0; i < D / 32; ++i)
      kt.k[r][i] = tok < tend ? ldg_stream_u4(p + 8 * i) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int tok = tok0 + (r >> 1) * 8 + 2 * tq + (r & 1);
    const T* p = vbase + static_cast<int64_t>(tok) * sv_s + (D / 8) * g;
#pragma unroll
    for (int i = 0; i < D / 64; ++i)
      kt.v[r][i] = tok < tend ? ldg_stream_u4(p + 8 * i) : make_uint4(0, 0, 0, 0);
  }
}

// Physical 16-byte chunk of logical chunk c (4 floats of O) in a row of the cross-warp staging
// buffer. Thread t writes logical chunks [t*D/16, (t+1)*D/16); the XOR spreads the 8 threads of a
// quarter-warp (rows 2q, 2q+1 x t = 0..3) over 8 distinct chunk positions modulo 8, so the 16-byte
// stores and the merge loop's 4-byte reads are free of bank conflicts.
template <int D>
__device__ __forceinline__ int o_chunk(int row, int c) {
  if (D == 128) {
    const int t = c >> 3;
    return (t << 3) | ((c & 7) ^ ((t + 4 * (row & 1)) & 7));
  } else {
    const int t = c >> 2;
    return (t << 2) | ((c & 3) ^ (((t >> 1) + 2 * (row & 1)) & 3));
  }
}

// Single-launch mode (both partial kernels): after a split CTA has written its partial, the last of the
// sequence's valid splits to arrive combines them. The barrier orders every thread's partial stores
// before thread 0's release; thread 0's acquire (and the barrier after it) orders the reads below after
// every other split's partial. The counter returns to zero for the next launch.
template <typename T, int D>
__device__ __forceinline__ void last_split_combine(const AttnArgs& a, int b, int kvh, int len) {
  __shared__ int s_last;
  const int nvalid = min(a.nsplit, (len + a.chunk - 1) / a.chunk);
  __syncthreads();
  if (threadIdx.x == 0) {
    int* ctr = a.counters + b * a.KVH + kvh;
    const int last = atomic_add_acq_rel_gpu(ctr, 1) == nvalid - 1;
    if (last) *ctr = 0;   // every split has arrived: reset for the next launch
    s_last = last;
  }
  __syncthreads();
  if (!s_last) return;
  const int64_t head0 = static_cast<int64_t>(b) * a.H + kvh * a.G;
  for (int idx = threadIdx.x; idx < a.G * D; idx += kAttnWarps * 32) {
    const int row = idx / D, d = idx - row * D;
    const int64_t base = (head0 + row) * a.nsplit;
    float mx = -INFINITY;
    for (int i = 0; i < nvalid; ++i) mx = fmaxf(mx, __ldcg(a.ml + (base + i) * 2));
    float num = 0.f, den = 0.f;
    for (int i = 0; i < nvalid; ++i) {
      const float m = __ldcg(a.ml + (base + i) * 2);
      const float w = m == -INFINITY ? 0.f : exp2f(m - mx);
      num += w * __ldcg(a.acc + (base + i) * D + d);
      den += w * __ldcg(a.ml + (base + i) * 2 + 1);
    }
    store_out<T>(a, b, kvh * a.G + row, d, den > 0.f ? num / den : 0.f);
  }
}

template <typename T, int D, bool TWO_HALVES>
__global__ void __launch_bounds__(kAttnWarps * 32, 2) gqa_partial_kernel(const AttnArgs a) {
  constexpr int KSTEPS = D / 16;   // MMA k-steps over the head dim
  constexpr int NTILES = D / 8;    // n8 output tiles of O
  constexpr int ROWS = TWO_HALVES ? 16 : 8;
  __shared__ __align__(16) float s_o[kAttnWarps][ROWS][D];   // 16-byte chunks swizzled by o_chunk()
  __shared__ float s_m[kAttnWarps][ROWS], s_l[kAttnWarps][ROWS];

  pdl_wait();   // no-op unless launched as a programmatic dependent
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int len = seqlen_of(a, b);
  const int t_begin = split * a.chunk;
  if (t_begin >= len) {   // this split holds no keys; the combine skips it
    if (a.fused && split == 0)   // an empty sequence: its heads get zeros, as the combine kernel writes
      for (int idx = threadIdx.x; idx < a.G * D; idx += kAttnWarps * 32)
        store_out<T>(a, b, kvh * a.G + idx / D, idx % D, 0.f);
    return;
  }
  const int t_end = min(t_begin + a.chunk, len);

  // ---- Q fragments (rows = heads of this KV group), permuted head-dim order
  const T* qb = static_cast<const T*>(a.q) + b * a.sq_b;
  uint32_t qa[KSTEPS][4];
  {
    const int h0 = kvh * a.G + g, h1 = kvh * a.G + g + 8;
    const T* q0 = qb + static_cast<int64_t>(h0) * a.sq_h + (D / 4) * tq;
    const T* q1 = qb + static_cast<int64_t>(h1) * a.sq_h + (D / 4) * tq;
#pragma unroll
    for (int i = 0; i < D / 32; ++i) {
      const uint4 u0 = g < a.G ? __ldg(reinterpret_cast<const uint4*>(q0) + i) : make_uint4(0, 0, 0, 0);
      uint4 u1 = make_uint4(0, 0, 0, 0);
      if (TWO_HALVES && g + 8 < a.G) u1 = __ldg(reinterpret_cast<const uint4*>(q1) + i);
      // k-steps 2i and 2i+1 take the 8 halves of this uint4: a0/a2 = (d, d+1)/(d+2, d+3)
      qa[2 * i][0] = u0.x; qa[2 * i][2] = u0.y; qa[2 * i + 1][0] = u0.z; qa[2 * i + 1][2] = u0.w;
      qa[2 * i][1] = u1.x; qa[2 * i][3] = u1.y; qa[2 * i + 1][1] = u1.z; qa[2 * i + 1][3] = u1.w;
    }
  }

  const T* kbase = static_cast<const T*>(a.k) + b * a.sk_b + kvh * a.sk_h;
  const T* vbase = static_cast<const T*>(a.v) + b * a.sv_b + kvh * a.sv_h;

  float o[NTILES][4];
#pragma unroll
  for (int n = 0; n < NTILES; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};   // rows g, g+8 (log2 domain)
  float l_run[2] = {0.f, 0.f};               // per-thread partial sums over its keys

  const int ntiles = (t_end - t_begin + 15) / 16;
  KvTile<T, D> cur, nxt;
  int tile = warp;
  if (tile < ntiles) load_tile<T, D>(cur, kbase, vbase, a.sk_s, a.sv_s, t_begin + 16 * tile, t_end, g, tq);
  for (; tile < ntiles; tile += kAttnWarps) {
    const int tok0 = t_begin + 16 * tile;
    if (tile + kAttnWarps < ntiles)
      load_tile<T, D>(nxt, kbase, vbase, a.sk_s, a.sv_s, tok0 + 16 * kAttnWarps, t_end, g, tq);

    // S for keys tok0+[0,8) (s0) and tok0+[8,16) (s1)
    float s[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      s[h][0] = s[h][1] = s[h][2] = s[h][3] = 0.f;
#pragma unroll
      for (int j = 0; j < KSTEPS; ++j) {
        const uint32_t* kw = reinterpret_cast<const uint32_t*>(&cur.k[h][0]);
        Mma<T>::run(s[h], qa[j][0], qa[j][1], qa[j][2], qa[j][3], kw[2 * j], kw[2 * j + 1]);
      }
    }
    // scale, mask, online softmax
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int tok = tok0 + h * 8 + 2 * tq + (c & 1);
        s[h][c] = tok < t_end ? s[h][c] * a.scale_log2 : -INFINITY;
        tmax[c >> 1] = fmaxf(tmax[c >> 1], s[h][c]);
      }
    }
    float alpha[2], msafe[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 1));
      tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 2));
      const float m_new = fmaxf(m_run[r], tmax[r]);
      msafe[r] = m_new == -INFINITY ? 0.f : m_new;
      alpha[r] = exp2f(m_run[r] - msafe[r]);
      m_run[r] = m_new;
    }
    uint32_t pa[4];
    {
      float p[2][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 4; ++c) p[h][c] = exp2f(s[h][c] - msafe[c >> 1]);
      l_run[0] = l_run[0] * alpha[0] + (p[0][0] + p[0][1] + p[1][0] + p[1][1]);
      l_run[1] = l_run[1] * alpha[1] + (p[0][2] + p[0][3] + p[1][2] + p[1][3]);
      pa[0] = Dt<T>::pack2(p[0][0], p[0][1]);   // row g,   keys 2t, 2t+1
      pa[1] = Dt<T>::pack2(p[0][2], p[0][3]);   // row g+8
      pa[2] = Dt<T>::pack2(p[1][0], p[1][1]);   // row g,   keys 8+2t, 9+2t
      pa[3] = Dt<T>::pack2(p[1][2], p[1][3]);
    }
    // O = alpha*O + P V
    const uint32_t* v0 = reinterpret_cast<const uint32_t*>(&cur.v[0][0]);
    const uint32_t* v1 = reinterpret_cast<const uint32_t*>(&cur.v[1][0]);
    const uint32_t* v2 = reinterpret_cast<const uint32_t*>(&cur.v[2][0]);
    const uint32_t* v3 = reinterpret_cast<const uint32_t*>(&cur.v[3][0]);
#pragma unroll
    for (int n = 0; n < NTILES; ++n) {
      o[n][0] *= alpha[0]; o[n][1] *= alpha[0];
      o[n][2] *= alpha[1]; o[n][3] *= alpha[1];
      const uint32_t sel = (n & 1) ? 0x7632u : 0x5410u;
      const uint32_t b0 = __byte_perm(v0[n >> 1], v1[n >> 1], sel);
      const uint32_t b1 = __byte_perm(v2[n >> 1], v3[n >> 1], sel);
      Mma<T>::run(o[n], pa[0], pa[1], pa[2], pa[3], b0, b1);
    }
    if (tile + kAttnWarps < ntiles) cur = nxt;
  }

  // ---- per-warp results -> shared memory (rows g, g+8; thread owns d in [D/4*t, D/4*t + D/4))
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
#pragma unroll
  for (int r = 0; r < (TWO_HALVES ? 2 : 1); ++r) {
    const int row = g + 8 * r;
    if (tq == 0) {
      s_m[warp][row] = m_run[r];
      s_l[warp][row] = l_run[r];
    }
    // the thread's D/4 columns [D/4*t, D/4*t + D/4) as D/16 float4 chunks: o[n][2r] fill the first
    // half (n = 0..D/8-1), o[n][2r+1] the second
    float4* dst = reinterpret_cast<float4*>(&s_o[warp][row][0]);
#pragma unroll
    for (int i = 0; i < D / 16; ++i) {
      const int n0 = (i % (D / 32)) * 4, c = 2 * r + i / (D / 32);
      dst[o_chunk<D>(row, (D / 16) * tq + i)] = make_float4(o[n0][c], o[n0 + 1][c], o[n0 + 2][c], o[n0 + 3][c]);
    }
  }
  __syncthreads();

  // ---- merge the warps and write this split's partial
  const int nrows = min(a.G, ROWS);
  const int64_t slot0 = (static_cast<int64_t>(b) * a.H + kvh * a.G) * a.nsplit + split;
  for (int idx = threadIdx.x; idx < nrows * D; idx += kAttnWarps * 32) {
    const int row = idx / D, d = idx - row * D;
    float mx = s_m[0][row];
#pragma unroll
    for (int w = 1; w < kAttnWarps; ++w) mx = fmaxf(mx, s_m[w][row]);
    float acc = 0.f, l = 0.f;
    const int phys = o_chunk<D>(row, d >> 2) * 4 + (d & 3);
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float e = s_m[w][row] == -INFINITY ? 0.f : exp2f(s_m[w][row] - mx);
      acc += e * s_o[w][row][phys];
      l += e * s_l[w][row];
    }
    const int64_t slot = slot0 + static_cast<int64_t>(row) * a.nsplit;
    a.acc[slot * D + d] = acc;
    if (d == 0) {
      a.ml[slot * 2] = mx;
      a.ml[slot * 2 + 1] = l;
    }
  }
  pdl_launch_dependents();
  if (a.fused) last_split_combine<T, D>(a, b, kvh, len);
}

// One CTA per (b, h), one thread per head-dim element. OT: output dtype.
template <typename OT, int D>
__global__ void __launch_bounds__(D) gqa_combine_kernel(const AttnArgs a) {
  pdl_launch_dependents();   // the next kernel (o_proj) may start its weight prefetch
  pdl_wait();                // partial results of the previous kernel are visible after this
  const int bh = blockIdx.x;
  const int b = bh / a.H, h = bh - b * a.H;
  const int d = threadIdx.x;
  const int len = seqlen_of(a, b);
  const int nvalid = min(a.nsplit, (len + a.chunk - 1) / a.chunk);
  const int64_t base = static_cast<int64_t>(bh) * a.nsplit;
  float mx = -INFINITY;
  for (int i = 0; i < nvalid; ++i) mx = fmaxf(mx, a.ml[(base + i) * 2]);
  float num = 0.f, den = 0.f;
  for (int i = 0; i < nvalid; ++i) {
    const float m = a.ml[(base + i) * 2];
    const float w = m == -INFINITY ? 0.f : exp2f(m - mx);
    num += w * a.acc[(base + i) * D + d];
    den += w * a.ml[(base + i) * 2 + 1];
  }
  OT* out = static_cast<OT*>(a.out) + b * a.so_b + h * a.so_h;
  out[d] = Dt<OT>::from_f32(den > 0.f ? num / den : 0.f);
}

// ------------------------------------------------------------------------------------------------
// Streaming variant of the partial kernel (the default for two-kernel launches): the same CTA grid, split
// and workspace format, with K and V staged through shared memory so that far more bytes are in flight.
//  * A stage is 64 keys of K and of V (32 KB at D = 128), copied by every thread with 16-byte cp.async
//    (16 threads per 256-byte key row: whole lines), keys past the split's end zero-filled without a
//    global read. Three stages per CTA, two CTAs per SM: up to 128 KB in flight per SM.
//  * 16-byte chunk c of key row r sits at chunk c ^ (r & 7), so the ldmatrix reads below (8 key rows of
//    one chunk column at a time) hit 8 distinct bank groups.
//  * Warp w takes keys [16w, 16w + 16) of each stage. S = Q K^T: Q (the G heads as MMA rows) in
//    registers in natural head-dim order, K as the B operand by ldmatrix.x4 (rows = keys, two k-steps of
//    one 8-key tile per instruction). O += P V: P from the S accumulator, V as the B operand by
//    ldmatrix.x4.trans (two 8-column d tiles per instruction). Online softmax in the log2 domain as in the
//    register kernel; the warps meet in shared memory at the end and write one partial per split.
constexpr int kStreamKeys = 64;
constexpr int kStreamStages = 3;

__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr) : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr) : "memory");
}

// Coherent 4-byte load in volatile asm (data of the preceding kernel: stays below the dependency wait).
__device__ __forceinline__ uint32_t ld_act_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
template <typename T>
__device__ __forceinline__ float rnd16(float v) { return Dt<T>::to_f32(Dt<T>::from_f32(v)); }
// RoPE of two element pairs (x1 = lo[e] at d, x2 = hi[e] at d + D/2) with the rounding of the rotary
// kernel (q * cos + rotate_half(q) * sin, every product rounded to T, the sum rounded to T).
template <typename T>
__device__ __forceinline__ void rope_pair(uint32_t& lo, uint32_t& hi, uint32_t c1, uint32_t c2, uint32_t s1,
                                          uint32_t s2) {
  const T* xl = reinterpret_cast<const T*>(&lo);
  const T* xh = reinterpret_cast<const T*>(&hi);
  const T* pc1 = reinterpret_cast<const T*>(&c1);
  const T* pc2 = reinterpret_cast<const T*>(&c2);
  const T* ps1 = reinterpret_cast<const T*>(&s1);
  const T* ps2 = reinterpret_cast<const T*>(&s2);
  float o1[2], o2[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float x1 = Dt<T>::to_f32(xl[e]), x2 = Dt<T>::to_f32(xh[e]);
    o1[e] = rnd16<T>(x1 * Dt<T>::to_f32(pc1[e])) + rnd16<T>(-x2 * Dt<T>::to_f32(ps1[e]));
    o2[e] = rnd16<T>(x2 * Dt<T>::to_f32(pc2[e])) + rnd16<T>(x1 * Dt<T>::to_f32(ps2[e]));
  }
  lo = Dt<T>::pack2(o1[0], o1[1]);
  hi = Dt<T>::pack2(o2[0], o2[1]);
}

template <int D>
constexpr size_t stream_smem_bytes() {
  return static_cast<size_t>(kStreamStages) * 2 * kStreamKeys * D * 2;
}

// This CTA's share of the launch's L2 prefetch ranges: slice `cta` of each range (16-byte multiples), in
// bulk prefetches of at most 64 KB. One thread issues them; they complete on their own.
__device__ __forceinline__ void l2_prefetch_slices(const AttnArgs& a) {
  const int64_t ncta = static_cast<int64_t>(gridDim.x) * gridDim.y * gridDim.z;
  const int64_t cta = blockIdx.x + static_cast<int64_t>(gridDim.x) * (blockIdx.y + static_cast<int64_t>(gridDim.y) * blockIdx.z);
  for (int r = 0; r < a.npf && r < kMaxL2Prefetch; ++r) {
    const int64_t per = ((a.pf_bytes[r] + ncta - 1) / ncta + 15) & ~static_cast<int64_t>(15);
    const int64_t end = min(a.pf_bytes[r], (cta + 1) * per);
    for (int64_t o = cta * per; o < end; o += 65536) {
      const uint32_t n = static_cast<uint32_t>(end - o < 65536 ? end - o : 65536);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.pf_base[r] + o), "r"(n) : "memory");
    }
  }
}

template <typename T, int D, bool TWO_HALVES>
__global__ void __launch_bounds__(kAttnWarps * 32, 2) gqa_stream_kernel(const AttnArgs a) {
  constexpr int KSTEPS = D / 16;        // MMA k-steps over the head dim (S = Q K^T)
  constexpr int NTILES = D / 8;         // n8 output tiles of O
  constexpr int CH = D / 8;             // 16-byte chunks per key row
  constexpr uint32_t ROWB = D * 2;      // bytes per key row
  constexpr uint32_t TILEB = kStreamKeys * ROWB;   // K (or V) bytes of one stage
  constexpr int ROWS = TWO_HALVES ? 16 : 8;
  constexpr int OPAD = D + 8;           // merge-buffer row stride in floats (spreads rows over the banks)
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float s_m[kAttnWarps][ROWS], s_l[kAttnWarps][ROWS];

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int t_begin = split * a.chunk;
  const T* kbase = static_cast<const T*>(a.k) + b * a.sk_b + kvh * a.sk_h;
  const T* vbase = static_cast<const T*>(a.v) + b * a.sv_b + kvh * a.sv_h;
  const uint32_t sbase = smem_u32(smem);
  if (a.npf > 0 && tid == 0) l2_prefetch_slices(a);

  // copies of stage `it` into buffer `bf` (every thread: 64 keys x CH chunks of K and of V); keys at or
  // past `lim` are zero-filled without a global read
  auto issue = [&](int it, int bf, int lim) {
    const uint32_t kdst = sbase + static_cast<uint32_t>(bf) * 2 * TILEB, vdst = kdst + TILEB;
    const int t0 = t_begin + it * kStreamKeys;
#pragma unroll
    for (int i = 0; i < kStreamKeys * CH / (kAttnWarps * 32); ++i) {
      const int ci = tid + i * kAttnWarps * 32;
      const int r = ci / CH, c = ci % CH;
      const int tok = t0 + r;
      const bool ok = tok < lim;
      const int tk = ok ? tok : t_begin;
      const uint32_t off = static_cast<uint32_t>(r) * ROWB + static_cast<uint32_t>((c ^ (r & 7)) * 16);
      cp_async16_zfill(kdst + off, kbase + static_cast<int64_t>(tk) * a.sk_s + c * 8, ok);
      cp_async16_zfill(vdst + off, vbase + static_cast<int64_t>(tk) * a.sv_s + c * 8, ok);
    }
  };
  // With a static prefix (a decode step's append writes only each sequence's newest key/value), whole
  // stages below the newest key start before the dependency wait. The length read here may be this step's
  // or the previous one's (the appending kernel may not have written it yet): both bound keys that no
  // preceding kernel writes. In append mode the position comes from pos[b], written before the step.
  int pre = 0;
  int64_t apos = -1;   // append mode: this step's position of sequence b
  if (a.append) {
    apos = a.pos[b];
    if (apos < 0 || apos >= a.S) apos = -1;
  }
  if (a.kv_prefix || a.append) {
    int seen = a.S;
    if (a.append) {
      seen = static_cast<int>(apos) + 1;   // 0 for an invalid position
    } else if (a.seqlens) {
      asm volatile("ld.volatile.global.s32 %0, [%1];\n" : "=r"(seen) : "l"(a.seqlens + b) : "memory");
      seen = seen < 0 ? 0 : (seen > a.S ? a.S : seen);
    }
    const int lim = min(t_begin + a.chunk, seen - 1);
    while (pre < kStreamStages - 1 && t_begin + (pre + 1) * kStreamKeys <= lim) ++pre;
    for (int i = 0; i < pre; ++i) {
      issue(i, i, lim);
      cp_async_commit();
    }
  }
  pdl_wait();   // no-op unless launched as a programmatic dependent
  const int len = a.append ? static_cast<int>(apos) + 1 : seqlen_of(a, b);
  if (a.append && split == 0 && kvh == 0 && tid == 0) a.seqlens_out[b] = len;
  if (t_begin >= len) {   // this split holds no keys; the combine skips it
    cp_async_wait<0>();
    if (a.fused && split == 0)   // an empty sequence: its heads get zeros, as the combine kernel writes
      for (int idx = tid; idx < a.G * D; idx += kAttnWarps * 32) store_out<T>(a, b, kvh * a.G + idx / D, idx % D, 0.f);
    return;
  }
  const int t_end = min(t_begin + a.chunk, len);

  // ---- Q fragments (rows = heads of this KV group), natural head-dim order
  uint32_t qa[KSTEPS][4];
  {
    const T* qb = static_cast<const T*>(a.q) + b * a.sq_b;
    const int h0 = kvh * a.G + g, h1 = kvh * a.G + g + 8;
    const uint32_t* q0 = reinterpret_cast<const uint32_t*>(qb + static_cast<int64_t>(h0) * a.sq_h);
    const uint32_t* q1 = reinterpret_cast<const uint32_t*>(qb + static_cast<int64_t>(h1) * a.sq_h);
    const bool v0 = g < a.G, v1 = TWO_HALVES && g + 8 < a.G;
#pragma unroll
    for (int j = 0; j < KSTEPS; ++j) {
      qa[j][0] = v0 ? ld_act_u32(q0 + 8 * j + tq) : 0u;       // d = 16j + 2tq, +1
      qa[j][2] = v0 ? ld_act_u32(q0 + 8 * j + 4 + tq) : 0u;   // d = 16j + 8 + 2tq, +1
      qa[j][1] = v1 ? ld_act_u32(q1 + 8 * j + tq) : 0u;
      qa[j][3] = v1 ? ld_act_u32(q1 + 8 * j + 4 + tq) : 0u;
    }
    if (a.append) {
      // RoPE in registers, rounded as the rotary kernel rounds: d < D/2 pairs with d + D/2, and both sit in
      // this lane (k-steps j and j + KSTEPS/2 at the same fragment position)
      const uint32_t* cs = reinterpret_cast<const uint32_t*>(static_cast<const T*>(a.rcos) + apos * a.ld_cs);
      const uint32_t* sn = reinterpret_cast<const uint32_t*>(static_cast<const T*>(a.rsin) + apos * a.ld_cs);
#pragma unroll
      for (int j = 0; j < KSTEPS / 2; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int w = 8 * j + (r >= 2 ? 4 : 0) + tq;   // u32 index of this fragment's pair
          rope_pair<T>(qa[j][r], qa[j + KSTEPS / 2][r], __ldg(cs + w), __ldg(cs + w + D / 4), __ldg(sn + w),
                       __ldg(sn + w + D / 4));
        }
    }
  }
  if (a.append && t_begin <= len - 1 && len - 1 < t_end) {
    // this split holds the new position: rotate this step's key and append it and the value to the cache
    // before any stage that covers it is copied
    const int64_t p = len - 1;
    const T* kn = static_cast<const T*>(a.k_new) + b * a.ldk_new + static_cast<int64_t>(kvh) * D;
    const T* vn = static_cast<const T*>(a.v_new) + b * a.ldv_new + static_cast<int64_t>(kvh) * D;
    T* kd = const_cast<T*>(kbase) + p * a.sk_s;
    T* vd = const_cast<T*>(vbase) + p * a.sv_s;
    const T* cs = static_cast<const T*>(a.rcos) + p * a.ld_cs;
    const T* sn = static_cast<const T*>(a.rsin) + p * a.ld_cs;
    if (tid < D / 2) {
      const int i = tid;
      const float x1 = Dt<T>::to_f32(kn[i]), x2 = Dt<T>::to_f32(kn[i + D / 2]);
      const float c1 = Dt<T>::to_f32(cs[i]), c2 = Dt<T>::to_f32(cs[i + D / 2]);
      const float s1 = Dt<T>::to_f32(sn[i]), s2 = Dt<T>::to_f32(sn[i + D / 2]);
      kd[i] = Dt<T>::from_f32(rnd16<T>(x1 * c1) + rnd16<T>(-x2 * s1));
      kd[i + D / 2] = Dt<T>::from_f32(rnd16<T>(x2 * c2) + rnd16<T>(x1 * s2));
    } else if (tid < D) {
      const int i = 2 * (tid - D / 2);
      *reinterpret_cast<uint32_t*>(vd + i) = *reinterpret_cast<const uint32_t*>(vn + i);
    }
    __threadfence_block();
    __syncthreads();
  }
  const int nst = (t_end - t_begin + kStreamKeys - 1) / kStreamKeys;
  for (int i = pre; i < kStreamStages - 1; ++i) {
    if (i < nst) issue(i, i, t_end);
    cp_async_commit();
  }

  float o[NTILES][4];
#pragma unroll
  for (int n = 0; n < NTILES; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};   // rows g, g+8 (log2 domain)
  float l_run[2] = {0.f, 0.f};               // per-thread partial sums over its keys

  // ldmatrix lane roles: matrix mi = lane / 8, row ri = lane % 8
  const int mi = lane >> 3, ri = lane & 7;
  for (int it = 0; it < nst; ++it) {
    cp_async_wait<kStreamStages - 2>();   // this thread's copies of stage `it` have landed
    __syncthreads();                      // everyone's; and every warp is done with stage it - 1
    if (it + kStreamStages - 1 < nst) issue(it + kStreamStages - 1, (it + kStreamStages - 1) % kStreamStages, t_end);
    cp_async_commit();
    const int key0 = t_begin + it * kStreamKeys + 16 * warp;   // this warp's first key
    if (key0 >= t_end) continue;   // warp-uniform: all its keys are past the end
    const uint32_t kbuf = sbase + static_cast<uint32_t>(it % kStreamStages) * 2 * TILEB, vbuf = kbuf + TILEB;

    // S for keys key0 + [0, 8) (s[0]) and key0 + [8, 16) (s[1])
    float s[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      s[h][0] = s[h][1] = s[h][2] = s[h][3] = 0.f;
      const int r = 16 * warp + 8 * h + ri;   // key row in the stage
#pragma unroll
      for (int j = 0; j < KSTEPS; j += 2) {
        const int c = 2 * j + mi;   // chunks 2j, 2j+1 (k-step j), 2j+2, 2j+3 (k-step j+1)
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kbuf + static_cast<uint32_t>(r) * ROWB + static_cast<uint32_t>((c ^ (r & 7)) * 16), b0, b1, b2, b3);
        Mma<T>::run(s[h], qa[j][0], qa[j][1], qa[j][2], qa[j][3], b0, b1);
        Mma<T>::run(s[h], qa[j + 1][0], qa[j + 1][1], qa[j + 1][2], qa[j + 1][3], b2, b3);
      }
    }
    // scale, mask, online softmax
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int tok = key0 + h * 8 + 2 * tq + (c & 1);
        s[h][c] = tok < t_end ? s[h][c] * a.scale_log2 : -INFINITY;
        tmax[c >> 1] = fmaxf(tmax[c >> 1], s[h][c]);
      }
    }
    float alpha[2], msafe[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 1));
      tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 2));
      const float m_new = fmaxf(m_run[r], tmax[r]);
      msafe[r] = m_new == -INFINITY ? 0.f : m_new;
      alpha[r] = exp2f(m_run[r] - msafe[r]);
      m_run[r] = m_new;
    }
    uint32_t pa[4];
    {
      float p[2][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 4; ++c) p[h][c] = exp2f(s[h][c] - msafe[c >> 1]);
      l_run[0] = l_run[0] * alpha[0] + (p[0][0] + p[0][1] + p[1][0] + p[1][1]);
      l_run[1] = l_run[1] * alpha[1] + (p[0][2] + p[0][3] + p[1][2] + p[1][3]);
      pa[0] = Dt<T>::pack2(p[0][0], p[0][1]);   // row g,   keys 2t, 2t+1
      pa[1] = Dt<T>::pack2(p[0][2], p[0][3]);   // row g+8
      pa[2] = Dt<T>::pack2(p[1][0], p[1][1]);   // row g,   keys 8+2t, 9+2t
      pa[3] = Dt<T>::pack2(p[1][2], p[1][3]);
    }
    // O = alpha*O + P V; V tiles by ldmatrix.trans: matrices (d tile 2p + mi/2, key half mi%2)
#pragma unroll
    for (int n = 0; n < NTILES; ++n) {
      o[n][0] *= alpha[0]; o[n][1] *= alpha[0];
      o[n][2] *= alpha[1]; o[n][3] *= alpha[1];
    }
#pragma unroll
    for (int np = 0; np < NTILES; np += 2) {
      const int r = 16 * warp + 8 * (mi & 1) + ri, c = np + (mi >> 1);
      uint32_t v0, v1, v2, v3;
      ldsm_x4_t(vbuf + static_cast<uint32_t>(r) * ROWB + static_cast<uint32_t>((c ^ (r & 7)) * 16), v0, v1, v2, v3);
      Mma<T>::run(o[np], pa[0], pa[1], pa[2], pa[3], v0, v1);
      Mma<T>::run(o[np + 1], pa[0], pa[1], pa[2], pa[3], v2, v3);
    }
  }
  cp_async_wait<0>();
  __syncthreads();   // the stage buffers become the merge buffer

  // ---- per-warp results -> shared memory (rows g, g+8; thread owns d = 8n + 2t, +1)
  float* s_o = reinterpret_cast<float*>(smem);   // [kAttnWarps][ROWS][OPAD]
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
#pragma unroll
  for (int r = 0; r < (TWO_HALVES ? 2 : 1); ++r) {
    const int row = g + 8 * r;
    if (tq == 0) {
      s_m[warp][row] = m_run[r];
      s_l[warp][row] = l_run[r];
    }
    float* dst = s_o + (warp * ROWS + row) * OPAD + 2 * tq;
#pragma unroll
    for (int n = 0; n < NTILES; ++n)
      *reinterpret_cast<float2*>(dst + 8 * n) = make_float2(o[n][2 * r], o[n][2 * r + 1]);
  }
  __syncthreads();

  // ---- merge the warps and write this split's partial (a warp that saw no keys has m = -inf, l = 0)
  const int nrows = min(a.G, ROWS);
  const int64_t slot0 = (static_cast<int64_t>(b) * a.H + kvh * a.G) * a.nsplit + split;
  for (int idx = tid; idx < nrows * D; idx += kAttnWarps * 32) {
    const int row = idx / D, d = idx - row * D;
    float mx = s_m[0][row];
#pragma unroll
    for (int w = 1; w < kAttnWarps; ++w) mx = fmaxf(mx, s_m[w][row]);
    float acc = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float e = s_m[w][row] == -INFINITY ? 0.f : exp2f(s_m[w][row] - mx);
      acc += e * s_o[(w * ROWS + row) * OPAD + d];
      l += e * s_l[w][row];
    }
    const int64_t slot = slot0 + static_cast<int64_t>(row) * a.nsplit;
    a.acc[slot * D + d] = acc;
    if (d == 0) {
      a.ml[slot * 2] = mx;
      a.ml[slot * 2 + 1] = l;
    }
  }
  pdl_launch_dependents();
  if (a.fused) last_split_combine<T, D>(a, b, kvh, len);
}

int check_attn(int B, int H, int KVH, int S, int D, int dtype) {
  if (B < 0 || H < 0 || KVH < 0 || S < 0) return B2D_ERR_ARG;
  if (dtype != B2D_F16 && dtype != B2D_BF16) return B2D_ERR_DTYPE;
  if (D != 64 && D != 128) return B2D_ERR_SHAPE;
  if (KVH == 0 || H % KVH != 0 || H / KVH > 16) return B2D_ERR_SHAPE;
  return B2D_OK;
}

int fill_args(AttnArgs* a, const void* q, int64_t sq_b, int64_t sq_h, const void* k, int64_t sk_b, int64_t sk_h,
              int64_t sk_s, const void* v, int64_t sv_b, int64_t sv_h, int64_t sv_s, const int32_t* seqlens, int B,
              int H, int KVH, int S, int D, float scale, int nsplit, int chunk, const void* ws, size_t ws_bytes) {
  if (nsplit <= 0 || chunk <= 0 || chunk % 16 != 0) return B2D_ERR_SHAPE;
  if (static_cast<int64_t>(nsplit) * chunk < S) return B2D_ERR_SHAPE;
  if (!ws || ws_bytes < b2d_gqa_workspace_bytes(B, H, nsplit, D)) return B2D_ERR_WORKSPACE;
  if (!aligned(ws, 16)) return B2D_ERR_ALIGN;
  *a = AttnArgs{};
  a->q = q; a->sq_b = sq_b; a->sq_h = sq_h;
  a->k = k; a->sk_b = sk_b; a->sk_h = sk_h; a->sk_s = sk_s;
  a->v = v; a->sv_b = sv_b; a->sv_h = sv_h; a->sv_s = sv_s;
  a->seqlens = seqlens;
  a->B = B; a->H = H; a->KVH = KVH; a->S = S; a->G = KVH ? H / KVH : 1;
  a->scale_log2 = scale * kLog2e;
  a->nsplit = nsplit; a->chunk = chunk;
  a->counters = static_cast<int*>(const_cast<void*>(ws));
  a->acc = reinterpret_cast<float*>(static_cast<uint8_t*>(const_cast<void*>(ws)) + kAttnCounterBytes);
  a->ml = a->acc + static_cast<size_t>(B) * H * nsplit * D;
  return B2D_OK;
}

template <typename T, int D>
int launch_partial_t(const AttnArgs& a, cudaStream_t s, bool pdl) {
  const dim3 grid(a.nsplit, a.KVH, a.B);
  if (a.G > 8) return launch_kernel(gqa_partial_kernel<T, D, true>, grid, dim3(kAttnWarps * 32), 0, s, pdl, a);
  return launch_kernel(gqa_partial_kernel<T, D, false>, grid, dim3(kAttnWarps * 32), 0, s, pdl, a);
}

// Which partial kernel serves a two-kernel launch: B2D_ATTN_KERNEL=stream / reg in the environment selects
// the streaming or the register-prefetch kernel (read at every call, for comparisons); otherwise
// kStreamByDefault decides. Both kernels implement the single-launch combine.
constexpr bool kStreamByDefault = true;   // measured faster at every shape (B = 1, 8; S = 512 .. 32768)
bool stream_attn_enabled() {
  const char* v = std::getenv("B2D_ATTN_KERNEL");
  if (v && std::strcmp(v, "reg") == 0) return false;
  if (v && std::strcmp(v, "stream") == 0) return true;
  return kStreamByDefault;
}

template <typename T, int D, bool TWO>
int launch_stream_tt(const AttnArgs& a, cudaStream_t s, bool pdl) {
  auto kern = gqa_stream_kernel<T, D, TWO>;
  constexpr size_t smem = stream_smem_bytes<D>();
  static bool configured[64] = {false};   // per device; setting it twice is harmless
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return B2D_ERR_DEVICE;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) { set_cuda_error(e); return B2D_ERR_LAUNCH; }
    configured[dev] = true;
  }
  return launch_kernel(kern, dim3(a.nsplit, a.KVH, a.B), dim3(kAttnWarps * 32), smem, s, pdl, a);
}

template <typename T, int D>
int launch_stream_t(const AttnArgs& a, cudaStream_t s, bool pdl) {
  return a.G > 8 ? launch_stream_tt<T, D, true>(a, s, pdl) : launch_stream_tt<T, D, false>(a, s, pdl);
}

int launch_partial(const AttnArgs& a, int D, int dtype, cudaStream_t s, bool pdl = false) {
  if (stream_attn_enabled()) {
    if (dtype == B2D_F16) return D == 64 ? launch_stream_t<__half, 64>(a, s, pdl) : launch_stream_t<__half, 128>(a, s, pdl);
    return D == 64 ? launch_stream_t<__nv_bfloat16, 64>(a, s, pdl) : launch_stream_t<__nv_bfloat16, 128>(a, s, pdl);
  }
  if (dtype == B2D_F16) {
    if (D == 64) return launch_partial_t<__half, 64>(a, s, pdl);
    return launch_partial_t<__half, 128>(a, s, pdl);
  }
  if (D == 64) return launch_partial_t<__nv_bfloat16, 64>(a, s, pdl);
  return launch_partial_t<__nv_bfloat16, 128>(a, s, pdl);
}

template <typename T, int D>
int launch_combine_t(const AttnArgs& a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.B * a.H);
  cfg.blockDim = dim3(D);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gqa_combine_kernel<T, D>, a);
  if (e != cudaSuccess) { set_cuda_error(e); return B2D_ERR_LAUNCH; }
  return launch_status();
}

int launch_combine(const AttnArgs& a, int D, int out_dtype, cudaStream_t s, bool pdl) {
  if (out_dtype == B2D_F16) {
    if (D == 64) return launch_combine_t<__half, 64>(a, s, pdl);
    return launch_combine_t<__half, 128>(a, s, pdl);
  }
  if (out_dtype == B2D_BF16) {
    if (D == 64) return launch_combine_t<__nv_bfloat16, 64>(a, s, pdl);
    return launch_combine_t<__nv_bfloat16, 128>(a, s, pdl);
  }
  if (D == 64) return launch_combine_t<float, 64>(a, s, pdl);
  return launch_combine_t<float, 128>(a, s, pdl);
}

int check_strides(const void* q, int64_t sq_b, int64_t sq_h, const void* k, int64_t sk_b, int64_t sk_h, int64_t sk_s,
                  const void* v, int64_t sv_b, int64_t sv_h, int64_t sv_s) {
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16)) return B2D_ERR_ALIGN;
  if ((sq_b | sq_h | sk_b | sk_h | sk_s | sv_b | sv_h | sv_s) % 8 != 0) return B2D_ERR_ALIGN;
  return B2D_OK;
}

}  // namespace
}  // namespace b2d

using namespace b2d;

extern "C" int b2d_gqa_default_splits(int B, int KVH, int S) {
  DeviceInfo di;
  if (device_info(&di) != B2D_OK || B <= 0 || KVH <= 0 || S <= 0) return 1;
  // About 1.75 CTAs per SM in one wave: measured best on B200 for B in {1, 8} and S from 320 to
  // 32768 keys (fewer, longer splits beat more waves of short ones: each CTA has a fixed cost), with
  // at least 64 keys per split (128 from 2048 keys up).
  const int64_t pairs = static_cast<int64_t>(B) * KVH;
  const int64_t target = static_cast<int64_t>(di.sm_count) * 7 / 4;
  int64_t ns = target / pairs;
  const int64_t min_chunk = S >= 2048 ? 128 : 64;
  const int64_t max_ns = (S + min_chunk - 1) / min_chunk;
  if (ns > max_ns) ns = max_ns;
  if (ns < 1) ns = 1;
  // round chunk up to a multiple of 32 keys and recompute the split count
  int64_t chunk = (S + ns - 1) / ns;
  chunk = (chunk + 31) / 32 * 32;
  return static_cast<int>((S + chunk - 1) / chunk);
}

extern "C" size_t b2d_gqa_workspace_bytes(int B, int H, int nsplit, int D) {
  if (B <= 0 || H <= 0 || nsplit <= 0 || D <= 0) return 0;
  return kAttnCounterBytes + static_cast<size_t>(B) * H * nsplit * (D + 2) * sizeof(float);
}

static int default_chunk(int S, int nsplit) {
  int chunk = (S + nsplit - 1) / nsplit;
  return (chunk + 31) / 32 * 32;
}

extern "C" int b2d_gqa_decode_partial(const void* q, int64_t sq_b, int64_t sq_h, const void* k, int64_t sk_b,
                                      int64_t sk_h, int64_t sk_s, const void* v, int64_t sv_b, int64_t sv_h,
                                      int64_t sv_s, const int32_t* seqlens, int B, int H, int KVH, int S, int D,
                                      float scale, int nsplit, int chunk, int dtype, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  int st = check_attn(B, H, KVH, S, D, dtype);
  if (st != B2D_OK) return st;
  if (B == 0 || H == 0 || S == 0) return B2D_OK;
  if (!q || !k || !v) return B2D_ERR_ARG;
  if ((st = check_strides(q, sq_b, sq_h, k, sk_b, sk_h, sk_s, v, sv_b, sv_h, sv_s)) != B2D_OK) return st;
  DeviceInfo di;
  if ((st = device_info(&di)) != B2D_OK) return st;
  AttnArgs a;
  if ((st = fill_args(&a, q, sq_b, sq_h, k, sk_b, sk_h, sk_s, v, sv_b, sv_h, sv_s, seqlens, B, H, KVH, S, D, scale,
                      nsplit, chunk, workspace, workspace_bytes)) != B2D_OK)
    return st;
  if (nsplit > 65535 || KVH > 65535 || B > 65535) return B2D_ERR_SHAPE;
  return launch_partial(a, D, dtype, static_cast<cudaStream_t>(stream));
}

extern "C" int b2d_gqa_decode_combine(const int32_t* seqlens, int B, int H, int S, int D, int nsplit, int chunk,
                                      int out_dtype, const void* workspace, size_t workspace_bytes, void* out,
                                      int64_t so_b, int64_t so_h, void* stream) {
  if (B < 0 || H < 0 || S < 0) return B2D_ERR_ARG;
  if (out_dtype != B2D_F16 && out_dtype != B2D_BF16 && out_dtype != B2D_F32) return B2D_ERR_DTYPE;
  if (D != 64 && D != 128) return B2D_ERR_SHAPE;
  if (B == 0 || H == 0) return B2D_OK;
  if (!out) return B2D_ERR_ARG;
  int st;
  DeviceInfo di;
  if ((st = device_info(&di)) != B2D_OK) return st;
  AttnArgs a;
  if ((st = fill_args(&a, nullptr, 0, 0, nullptr, 0, 0, 0, nullptr, 0, 0, 0, seqlens, B, H, 1, S, D, 1.f,
                      nsplit, chunk, workspace, workspace_bytes)) != B2D_OK)
    return st;
  a.G = 1;
  a.out = out; a.so_b = so_b; a.so_h = so_h;
  return launch_combine(a, D, out_dtype, static_cast<cudaStream_t>(stream), false);
}

extern "C" int b2d_gqa_decode_ex(const void* q, int64_t sq_b, int64_t sq_h, const void* k, int64_t sk_b,
                                 int64_t sk_h, int64_t sk_s, const void* v, int64_t sv_b, int64_t sv_h, int64_t sv_s,
                                 const int32_t* seqlens, int B, int H, int KVH, int S, int D, float scale, int nsplit,
                                 int chunk, int dtype, void* workspace, size_t workspace_bytes, void* out,
                                 int64_t so_b, int64_t so_h, int out_dtype, int flags, void* stream) {
  int st = check_attn(B, H, KVH, S, D, dtype);
  if (st != B2D_OK) return st;
  if (out_dtype != dtype && out_dtype != B2D_F32) return B2D_ERR_DTYPE;
  if (B == 0 || H == 0) return B2D_OK;
  if (!out) return B2D_ERR_ARG;
  if (S == 0) return B2D_ERR_SHAPE;   // nothing to attend to
  if (!q || !k || !v) return B2D_ERR_ARG;
  if ((st = check_strides(q, sq_b, sq_h, k, sk_b, sk_h, sk_s, v, sv_b, sv_h, sv_s)) != B2D_OK) return st;
  DeviceInfo di;
  if ((st = device_info(&di)) != B2D_OK) return st;
  if (nsplit <= 0 && chunk <= 0) {
    nsplit = b2d_gqa_default_splits(B, KVH, S);
    chunk = default_chunk(S, nsplit);
    nsplit = (S + chunk - 1) / chunk;
  } else if (chunk <= 0) {
    chunk = default_chunk(S, nsplit);
  } else if (nsplit <= 0) {
    nsplit = (S + chunk - 1) / chunk;
  }
  AttnArgs a;
  if ((st = fill_args(&a, q, sq_b, sq_h, k, sk_b, sk_h, sk_s, v, sv_b, sv_h, sv_s, seqlens, B, H, KVH, S, D, scale,
                      nsplit, chunk, workspace, workspace_bytes)) != B2D_OK)
    return st;
  if (nsplit > 65535 || KVH > 65535 || B > 65535) return B2D_ERR_SHAPE;
  a.out = out; a.so_b = so_b; a.so_h = so_h;
  a.kv_prefix = (flags & B2D_KV_STATIC_PREFIX) ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((flags & B2D_ATTN_FUSED_COMBINE) && nsplit <= kMaxFusedSplits && B * KVH <= kMaxAttnCounters) {
    a.fused = 1;
    a.out_f32 = out_dtype == B2D_F32;
    return launch_partial(a, D, dtype, s, (flags & B2D_LAUNCH_PDL) != 0);
  }
  if ((st = launch_partial(a, D, dtype, s, (flags & B2D_LAUNCH_PDL) != 0)) != B2D_OK) return st;
  return launch_combine(a, D, out_dtype, s, true);
}

extern "C" int b2d_gqa_decode(const void* q, int64_t sq_b, int64_t sq_h, const void* k, int64_t sk_b, int64_t sk_h,
                              int64_t sk_s, const void* v, int64_t sv_b, int64_t sv_h, int64_t sv_s,
                              const int32_t* seqlens, int B, int H, int KVH, int S, int D, float scale, int nsplit,
                              int chunk, int dtype, void* workspace, size_t workspace_bytes, void* out, int64_t so_b,
                              int64_t so_h, int out_dtype, void* stream) {
  return b2d_gqa_decode_ex(q, sq_b, sq_h, k, sk_b, sk_h, sk_s, v, sv_b, sv_h, sv_s, seqlens, B, H, KVH, S, D, scale,
                           nsplit, chunk, dtype, workspace, workspace_bytes, out, so_b, so_h, out_dtype, 0, stream);
}

// ------------------------------------------------------------------------------------------------
// Decode-step attention with the step's RoPE and KV append folded in (no counterpart in the reference,
// whose decode step rotates and appends with torch ops before calling its attention kernel). One launch of
// the streaming partial kernel + the combine instead of the rotary/append kernel + both attention kernels.
// One-shot L2 prefetch hint for this host thread's next b2d_gqa_decode_append call (then cleared).
thread_local int t_npf = 0;
thread_local const char* t_pf_base[kMaxL2Prefetch];
thread_local int64_t t_pf_bytes[kMaxL2Prefetch];

extern "C" int b2d_l2_prefetch_hint(const void* const* ptrs, const int64_t* bytes, int n) {
  if (n < 0 || n > kMaxL2Prefetch || (n > 0 && (!ptrs || !bytes))) return B2D_ERR_ARG;
  t_npf = 0;
  for (int i = 0; i < n; ++i) {
    if (!ptrs[i] || bytes[i] < 0) return B2D_ERR_ARG;
    if (!aligned(ptrs[i], 16)) return B2D_ERR_ALIGN;
    t_pf_base[t_npf] = static_cast<const char*>(ptrs[i]);
    t_pf_bytes[t_npf] = bytes[i] & ~static_cast<int64_t>(15);   // whole 16-byte units inside the range
    ++t_npf;
  }
  return B2D_OK;
}

extern "C" int b2d_gqa_decode_append(const void* q, int64_t ldq, const void* k_new, int64_t ldk, const void* v_new,
                                     int64_t ldv, const int64_t* pos, const void* rcos, const void* rsin,
                                     int64_t ld_cs, void* k_cache, int64_t sk_b, int64_t sk_h, int64_t sk_s,
                                     void* v_cache, int64_t sv_b, int64_t sv_h, int64_t sv_s, int32_t* seqlens,
                                     int B, int H, int KVH, int S, int D, float scale, int dtype, void* workspace,
                                     size_t workspace_bytes, void* out, int64_t so_b, int64_t so_h, int out_dtype,
                                     int flags, void* stream) {
  int st = check_attn(B, H, KVH, S, D, dtype);
  if (st != B2D_OK) return st;
  if (out_dtype != dtype && out_dtype != B2D_F32) return B2D_ERR_DTYPE;
  if (B == 0 || H == 0) return B2D_OK;
  if (S == 0) return B2D_ERR_SHAPE;
  if (!q || !k_new || !v_new || !pos || !rcos || !rsin || !k_cache || !v_cache || !seqlens || !out) return B2D_ERR_ARG;
  if (ldq < static_cast<int64_t>(H) * D || ldk < static_cast<int64_t>(KVH) * D || ldv < static_cast<int64_t>(KVH) * D ||
      ld_cs < D)
    return B2D_ERR_SHAPE;
  if ((st = check_strides(q, ldq, D, k_cache, sk_b, sk_h, sk_s, v_cache, sv_b, sv_h, sv_s)) != B2D_OK) return st;
  if (!aligned(k_new, 4) || !aligned(v_new, 4) || !aligned(rcos, 4) || !aligned(rsin, 4) || (ldk | ldv | ld_cs) % 2)
    return B2D_ERR_ALIGN;
  DeviceInfo di;
  if ((st = device_info(&di)) != B2D_OK) return st;
  int nsplit = b2d_gqa_default_splits(B, KVH, S);
  const int chunk = default_chunk(S, nsplit);
  nsplit = (S + chunk - 1) / chunk;
  AttnArgs a;
  if ((st = fill_args(&a, q, ldq, D, k_cache, sk_b, sk_h, sk_s, v_cache, sv_b, sv_h, sv_s, seqlens, B, H, KVH, S, D,
                      scale, nsplit, chunk, workspace, workspace_bytes)) != B2D_OK)
    return st;
  if (nsplit > 65535 || KVH > 65535 || B > 65535) return B2D_ERR_SHAPE;
  a.out = out; a.so_b = so_b; a.so_h = so_h;
  a.append = 1;
  a.k_new = k_new; a.ldk_new = ldk;
  a.v_new = v_new; a.ldv_new = ldv;
  a.pos = pos;
  a.rcos = rcos; a.rsin = rsin; a.ld_cs = ld_cs;
  a.seqlens_out = seqlens;
  if ((flags & B2D_ATTN_FUSED_COMBINE) && nsplit <= kMaxFusedSplits && B * KVH <= kMaxAttnCounters) {
    a.fused = 1;
    a.out_f32 = out_dtype == B2D_F32;
  }
  a.npf = t_npf;
  for (int i = 0; i < t_npf; ++i) { a.pf_base[i] = t_pf_base[i]; a.pf_bytes[i] = t_pf_bytes[i]; }
  t_npf = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool pdl = (flags & B2D_LAUNCH_PDL) != 0;
  if (dtype == B2D_F16)
    st = D == 64 ? launch_stream_t<__half, 64>(a, s, pdl) : launch_stream_t<__half, 128>(a, s, pdl);
  else
    st = D == 64 ? launch_stream_t<__nv_bfloat16, 64>(a, s, pdl) : launch_stream_t<__nv_bfloat16, 128>(a, s, pdl);
  if (st != B2D_OK || a.fused) return st;
  return launch_combine(a, D, out_dtype, s, true);
}

// ------------------------------------------------------------------------------------------------
// Allocation-free variant of b2d_gqa_decode.
//
// Some callers cannot allocate device memory for the split-K partials: a serving process whose
// allocator reserved the whole device budget up front and accounts for every byte, or a plugin that
// lives inside another framework's memory pool and must not call cudaMalloc behind its back (a
// cudaMalloc there can also stall the device while the host waits). For them the partials live in
// this file-scope array instead of a caller workspace. Every GPU that loads the library holds the
// array until the process exits. Nothing in it needs to start at zero (each call writes every
// partial it later reads), but all calls on a device share it and keep the last call's contents, so
// two calls that overlap on the GPU (different streams, no ordering between them) race.
static constexpr size_t kGqaNoAllocScratchBytes = size_t(8) << 20;   // 8 MiB
static __device__ __align__(256) uint8_t b2d_gqa_noalloc_scratch[kGqaNoAllocScratchBytes];

namespace {
// Device address of the array, per device: looked up once under a lock; later calls (from any host
// thread) read it without locking.
std::atomic<void*> g_noalloc_scratch_ptr[64];
std::mutex g_noalloc_lookup_mutex;
}

extern "C" int b2d_gqa_decode_noalloc(const void* q, int64_t sq_b, int64_t sq_h, const void* k, int64_t sk_b,
                                      int64_t sk_h, int64_t sk_s, const void* v, int64_t sv_b, int64_t sv_h,
                                      int64_t sv_s, const int32_t* seqlens, int B, int H, int KVH, int S, int D,
                                      float scale, int nsplit, int chunk, int dtype, void* out, int64_t so_b,
                                      int64_t so_h, int out_dtype, void* stream) {
  int st = check_attn(B, H, KVH, S, D, dtype);
  if (st != B2D_OK) return st;
  if (B == 0 || H == 0) return B2D_OK;
  if (S == 0) return B2D_ERR_SHAPE;
  DeviceInfo di;
  if ((st = device_info(&di)) != B2D_OK) return st;
  // the same split choice as b2d_gqa_decode, resolved here to size the scratch
  if (nsplit <= 0 && chunk <= 0) {
    nsplit = b2d_gqa_default_splits(B, KVH, S);
    chunk = default_chunk(S, nsplit);
    nsplit = (S + chunk - 1) / chunk;
  } else if (chunk <= 0) {
    chunk = default_chunk(S, nsplit);
  } else if (nsplit <= 0) {
    nsplit = (S + chunk - 1) / chunk;
  }
  const size_t need = b2d_gqa_workspace_bytes(B, H, nsplit, D);
  if (need > kGqaNoAllocScratchBytes) {
    char msg[200];
    std::snprintf(msg, sizeof(msg),
                  "b2d_gqa_decode_noalloc: %zu bytes of split partials needed (B=%d H=%d nsplit=%d D=%d), "
                  "static scratch holds %zu; use fewer splits or b2d_gqa_decode with a workspace",
                  need, B, H, nsplit, D, kGqaNoAllocScratchBytes);
    set_error_text(msg);
    return B2D_ERR_WORKSPACE;
  }
  // The host sees only a stand-in for the array's name; the kernels need its device address. The
  // first call on each device (with that device current) looks it up once; make that first call
  // before any stream capture.
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    if (e != cudaSuccess) set_cuda_error(e);
    return B2D_ERR_DEVICE;
  }
  void* scratch = g_noalloc_scratch_ptr[dev].load(std::memory_order_acquire);
  if (!scratch) {
    std::lock_guard<std::mutex> lock(g_noalloc_lookup_mutex);
    scratch = g_noalloc_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (!scratch) {
      e = cudaGetSymbolAddress(&scratch, b2d_gqa_noalloc_scratch);
      if (e != cudaSuccess || scratch == nullptr) {
        set_cuda_error(e);
        return B2D_ERR_DEVICE;
      }
      g_noalloc_scratch_ptr[dev].store(scratch, std::memory_order_release);
    }
  }
  return b2d_gqa_decode(q, sq_b, sq_h, k, sk_b, sk_h, sk_s, v, sv_b, sv_h, sv_s, seqlens, B, H, KVH, S, D, scale,
                        nsplit, chunk, dtype, scratch, kGqaNoAllocScratchBytes, out, so_b, so_h, out_dtype, stream);
}
