// Shared helpers for the sm_100a decode kernels: dtype traits, tensor-core fragments,
// device-property cache and launch-status plumbing for the C ABI in include/b200decode.h.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "b200decode.h"

namespace b2d {

// ------------------------------------------------------------------ status helpers
void set_cuda_error(cudaError_t e);
void set_error_text(const char* text);    // message returned by b2d_last_cuda_error()
int launch_status();                      // cudaGetLastError -> B2D_OK / B2D_ERR_LAUNCH

struct DeviceInfo {
  int sm_count = 0;
  int max_smem_optin = 0;
  int cc_major = 0;
  int l2_bytes = 0;
};
// Properties of the current device (queried once per device). Returns B2D_OK or B2D_ERR_DEVICE.
int device_info(DeviceInfo* out);

// ------------------------------------------------------------------ dtype traits
template <typename T> struct Dt;
template <> struct Dt<__half> {
  static __device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f32(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ uint16_t bits_rn(float v) { return __half_as_ushort(__float2half_rn(v)); }
  static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct Dt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f32(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ uint16_t bits_rn(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }
  static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

template <> struct Dt<float> {
  static __device__ __forceinline__ float to_f32(float v) { return v; }
  static __device__ __forceinline__ float from_f32(float v) { return v; }
};

// ------------------------------------------------------------------ tensor-core fragments
// D = A(16x16, row) * B(16x8, col) + C, fp32 accumulate. Fragment ownership (lane = 4*g + t):
//   a0: (row g,   k 2t..2t+1)   a1: (row g+8, k 2t..2t+1)
//   a2: (row g,   k 2t+8..+9)   a3: (row g+8, k 2t+8..+9)
//   b0: (k 2t..2t+1, col g)     b1: (k 2t+8..+9, col g)
//   c0: (row g, col 2t)  c1: (row g, col 2t+1)  c2: (row g+8, col 2t)  c3: (row g+8, col 2t+1)
// Pure register computations (no memory side effects), so not volatile: the compiler may interleave
// independent accumulation chains.
template <typename T> struct Mma;
template <> struct Mma<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  // d = A*B (zero accumulator input)
  static __device__ __forceinline__ void run0(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
  }
};
template <> struct Mma<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ void run0(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
  }
};

// ------------------------------------------------------------------ memory helpers
// Streaming 8/16-byte loads of data read exactly once (weights, KV cache): skip L1 allocation.
// Not volatile: the data is read-only for the kernel's lifetime, so the loads may be scheduled freely.
__device__ __forceinline__ uint2 ldg_stream_u2(const void* p) {
  uint2 r;
  asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// Asynchronous global -> shared copies (completion tracked per thread with commit/wait groups).
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Thread-block clusters: this CTA's rank and the cluster's size, the cluster index and count (1-D
// grids), a full cluster barrier (release/acquire: shared-memory writes before it are visible to the
// other CTAs' reads after it), and reads of another CTA's shared memory (distributed shared memory).
__device__ __forceinline__ int cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return static_cast<int>(r);
}
__device__ __forceinline__ int cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;\n" : "=r"(r));
  return static_cast<int>(r);
}
__device__ __forceinline__ int cluster_index() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;\n" : "=r"(r));
  return static_cast<int>(r);
}
__device__ __forceinline__ int cluster_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;\n" : "=r"(r));
  return static_cast<int>(r);
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// Cluster barrier without memory ordering: only says that every thread of the cluster got here (used
// to keep a CTA's shared memory alive until remote readers, whose loaded values are already consumed,
// are done with it).
__device__ __forceinline__ void cluster_sync_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\nbarrier.cluster.wait.aligned;\n" ::: "memory");
}
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t local_addr, int rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(local_addr), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];\n"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(remote) : "memory");
  return v;
}

// Tensor-parallel all-reduce through peer memory, flag-in-word protocol: a 64-bit word carries 32
// bits of data (two fp16/bf16 values) in its low half and the call's epoch in its high half, written
// with one 64-bit store, so a reader that sees the epoch also sees the data. Every rank owns one buffer
// mapped by all peers; its words start at kArDataOff, laid out [2 epoch parities][world][words].
constexpr size_t kArDataOff = 512;
constexpr int kArMaxWorld = 8;
struct ArPeers {
  uint8_t* peer[kArMaxWorld];   // peer[p] = rank p's buffer as seen from this GPU
  int rank, world;
  int64_t words;                // words per rank slot
  const int64_t* step;          // device step counter: epoch = step * sites + site + 1
  int site, sites;
};
__device__ __forceinline__ uint32_t ar_epoch(const ArPeers& p) {
  return static_cast<uint32_t>(*p.step * p.sites + p.site + 1);
}
// Rank `src`'s slot for epoch e in the buffer of rank `dst`.
__device__ __forceinline__ uint64_t* ar_slot(const ArPeers& p, int dst, int src, uint32_t e) {
  return reinterpret_cast<uint64_t*>(p.peer[dst] + kArDataOff) + (static_cast<int64_t>(e & 1) * p.world + src) * p.words;
}
__device__ __forceinline__ void st_word(uint64_t* p, uint64_t v) {
  asm volatile("st.volatile.global.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_word(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.volatile.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void ld_word2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];\n" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Device-scope acquire-release atomic add (cheaper than a sequentially consistent fence + atomic):
// writes made before it by this thread, or by threads it synchronised with through a barrier, are
// visible to whoever observes the new value; reads after it see what earlier releasers published.
__device__ __forceinline__ int atomic_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], %2;\n" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
// Read-only loads that may hit L1 (activations reused by many warps).
__device__ __forceinline__ uint4 ldg_u4(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return __byte_perm(w, 0u, 0x4440u + i); }

// Programmatic dependent launch: let the next kernel in the stream start its prologue early /
// wait until the previous kernel's memory is visible.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Launch through cudaLaunchKernelEx, optionally as a programmatic dependent of the previous kernel
// in the stream (the kernel must then call pdl_wait() before it touches stream-ordered data).
template <typename... KArgs, typename... Args>
int launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                  Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return B2D_ERR_LAUNCH;
  }
  return launch_status();
}

}  // namespace b2d
