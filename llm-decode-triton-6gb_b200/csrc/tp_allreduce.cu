// One-shot all-reduce (sum) over NVLink peer memory for tensor-parallel decode (sm_100a).
//
// No counterpart in the reference (single GPU). Replaces the NCCL all-reduce of the partial hidden
// states after o_proj and down_proj: at decode sizes (B x hidden fp16, 64 KiB at B = 8) the cost is
// latency, so every rank pushes its slice straight into every peer's memory in one NVLink traversal
// and each rank sums the world's slices locally.
//
// Low-latency protocol without fences or flags: every 8-byte word carries two elements and the call's
// epoch (low 32 bits: the elements, high 32 bits: the epoch) and is written with one 64-bit store, so
// a reader that sees the epoch in a word also sees its data. Every rank owns one buffer of
// b2d_allreduce_buffer_bytes() with the same layout, mapped by every peer (peer_bufs[p] = rank p's
// buffer as seen from this GPU):
//   int32  epoch[kMaxBlocks]          this rank's call counter per CTA (never touched by peers)
//   int32  errors                     count of timed-out waits (0 in a healthy run)
//   uint64 data[2][world][n_max / 2]  data[e & 1][p] = peer p's words for epoch e
// CTA c: epoch e = ++epoch[c]; store its chunk of `in` as words into data[e & 1][rank] of every peer;
// then for each word of its chunk, poll (bounded) data[e & 1][p] here until it carries epoch e, and sum
// over p in rank order in fp32, one rounding -> out. All ranks produce identical bits. Two parities
// suffice: a rank cannot write epoch e + 2 into a peer before that peer has written e + 1, which it
// does only after its epoch-e sums are done (the kernels of one rank are ordered).
#include "common.cuh"

namespace b2d {
namespace {

constexpr int kMaxBlocks = 64;
constexpr int kMaxWorld = 8;
constexpr int kArThreads = 256;
constexpr int kChunk = 4096;                 // elements per CTA
constexpr long long kSpinLimit = 1LL << 22;  // polls before a thread gives up on its peers (about a second)

struct ArArgs {
  const void* in;
  void* out;
  int64_t n, n_max;
  int rank, world, nblocks;
  uint8_t* peer[kMaxWorld];
};

__host__ __device__ inline size_t ar_data_off() { return kArDataOff; }

template <typename T>
__global__ void __launch_bounds__(kArThreads) allreduce_push_kernel(const ArArgs a) {
  pdl_launch_dependents();
  __shared__ int s_epoch;
  const int c = blockIdx.x, tid = threadIdx.x;
  uint8_t* mine = a.peer[a.rank];
  pdl_wait();   // `in` is the previous kernel's output; the previous call's epoch update is visible
  if (tid == 0) {
    int* ep = reinterpret_cast<int*>(mine) + c;
    s_epoch = *ep + 1;
    *ep = s_epoch;
  }
  __syncthreads();
  const uint32_t e = static_cast<uint32_t>(s_epoch);
  const int64_t w_lo = static_cast<int64_t>(c) * (kChunk / 2);            // word range of this chunk
  const int64_t w_hi = (c + 1) * static_cast<int64_t>(kChunk / 2) < a.n / 2 ? (c + 1) * static_cast<int64_t>(kChunk / 2) : a.n / 2;
  const int64_t words = a.n_max / 2;
  const size_t par = ar_data_off() + static_cast<size_t>(e & 1) * a.world * words * 8;
  const uint32_t* src = static_cast<const uint32_t*>(a.in);
  // push: one 64-bit store per word to every peer
  for (int64_t w = w_lo + tid; w < w_hi; w += kArThreads) {
    const uint64_t v = (static_cast<uint64_t>(e) << 32) | __ldg(src + w);
    for (int p = 0; p < a.world; ++p)
      st_word(reinterpret_cast<uint64_t*>(a.peer[p] + par) + static_cast<int64_t>(a.rank) * words + w, v);
  }
  // gather: poll each word of every peer until it carries this epoch, sum in rank order
  const uint64_t* base = reinterpret_cast<const uint64_t*>(mine + par);
  uint32_t* out = static_cast<uint32_t*>(a.out);
  // after a recorded timeout, later calls poll once and return (a missing peer costs one timeout)
  long long budget = *reinterpret_cast<volatile int*>(mine + 256) == 0 ? kSpinLimit : 0;
  for (int64_t w = w_lo + tid; w < w_hi; w += kArThreads) {
    float s0 = 0.f, s1 = 0.f;
    for (int p = 0; p < a.world; ++p) {
      const uint64_t* q = base + static_cast<int64_t>(p) * words + w;
      uint64_t v = ld_word(q);
      while (static_cast<uint32_t>(v >> 32) != e && budget > 0) {
        if (--budget == 0) atomicAdd(reinterpret_cast<int*>(mine) + kMaxBlocks, 1);
        v = ld_word(q);
      }
      const uint32_t d = static_cast<uint32_t>(v);
      const T* h = reinterpret_cast<const T*>(&d);
      s0 += Dt<T>::to_f32(h[0]);
      s1 += Dt<T>::to_f32(h[1]);
    }
    out[w] = Dt<T>::pack2(s0, s1);
  }
}

}  // namespace
}  // namespace b2d

using namespace b2d;

extern "C" size_t b2d_allreduce_buffer_bytes(int64_t n_max, int world, int dtype) {
  if (n_max <= 0 || world < 1 || world > kMaxWorld || (dtype != B2D_F16 && dtype != B2D_BF16)) return 0;
  return ar_data_off() + static_cast<size_t>(2) * world * (n_max / 2) * 8;
}

extern "C" int b2d_allreduce(const void* in, void* out, int64_t n, int dtype, void* const* peer_bufs, int rank,
                             int world, int64_t n_max, int flags, void* stream) {
  if (n < 0 || world < 1 || world > kMaxWorld || rank < 0 || rank >= world || n > n_max) return B2D_ERR_ARG;
  if (dtype != B2D_F16 && dtype != B2D_BF16) return B2D_ERR_DTYPE;
  if (n % 8 != 0 || n_max % 8 != 0 || (n + kChunk - 1) / kChunk > kMaxBlocks) return B2D_ERR_SHAPE;
  if (n == 0) return B2D_OK;
  if (!in || !out || !peer_bufs) return B2D_ERR_ARG;
  if (!aligned(in, 16) || !aligned(out, 16)) return B2D_ERR_ALIGN;
  ArArgs a{};
  a.in = in; a.out = out; a.n = n; a.n_max = n_max;
  a.rank = rank; a.world = world;
  a.nblocks = static_cast<int>((n + kChunk - 1) / kChunk);
  for (int p = 0; p < world; ++p) {
    if (!peer_bufs[p] || !aligned(peer_bufs[p], 256)) return B2D_ERR_ALIGN;
    a.peer[p] = static_cast<uint8_t*>(peer_bufs[p]);
  }
  DeviceInfo di;
  int st;
  if ((st = device_info(&di)) != B2D_OK) return st;
  const bool pdl = (flags & B2D_LAUNCH_PDL) != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B2D_F16)
    return launch_kernel(allreduce_push_kernel<__half>, dim3(a.nblocks), dim3(kArThreads), 0, s, pdl, a);
  return launch_kernel(allreduce_push_kernel<__nv_bfloat16>, dim3(a.nblocks), dim3(kArThreads), 0, s, pdl, a);
}
