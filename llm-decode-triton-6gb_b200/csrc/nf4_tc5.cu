// Fused NF4 dequant + GEMM on the 5th-generation tensor cores (tcgen05) for 9..64 tokens: the
// tensor-parallel batch-64 decode and other mid-sized batches. y[M, N] = x[M, K] @ W[N, K]^T with W in
// bitsandbytes NF4 (the reference's Triton kernel, profiling/kernels/nf4_gemm.py:37-64, serves at most
// 8 rows; above that the reference falls back to bitsandbytes' dequant + matmul, patch.py:36-40).
//
// At 64 tokens the product has ~250 flop per weight byte, near the B200 ridge, so the multiply belongs
// on tcgen05 while the dequant stays on the CUDA cores:
//  * CTA tile: 128 weight rows (the MMA's M) x all tokens padded to a multiple of 16 (the MMA's N) x a
//    range of K. The fp32 accumulator lives in tensor memory (TMEM: 128 lanes = rows, N columns).
//  * Warp 8 (one elected thread) streams the packed weights (boxes of 128 rows x 128 bytes = 4 blocks of
//    64 weights) and the activations (boxes of N tokens x 64 k) into a 2-stage shared-memory ring with
//    tensor copies (128-byte swizzle, no multicast), and issues the MMAs: tcgen05.mma kind::f16,
//    M=128, N=tokens, K=16, both operands K-major in shared memory, completion through tcgen05.commit
//    on mbarriers.
//  * Warps 0-7 (threads t and t + 128 = the two halves of tile row t) dequantise one block of 64 weights
//    at a time into a double-
//    buffered fp16/bf16 A tile in the canonical K-major 128-byte-swizzled layout: per packed byte one
//    byte permute + one shared table load (256 entries x 32 lane copies of the pair (code[hi],
//    code[lo]); conflict-free), one paired multiply by the block scale, one 16-byte store per 8 weights
//    (conflict-free under the swizzle). The A tile then feeds four MMAs.
//  * The weight tile is code * scale rounded to the activation dtype before the MMA (the scale cannot be
//    factored out of a tensor-memory accumulator), so products round once more than the M <= 8 kernel's.
//  * K split: clusters of 1, 2 or 4 CTAs split K; their partial tiles meet through distributed shared
//    memory in rank order (deterministic). Epilogue: tcgen05.ld of each warp's 32 TMEM lanes.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <type_traits>

#include "nf4_tc5.cuh"

namespace b2d {
namespace {

constexpr int kRows = 128;            // weight rows per tile (MMA M)
constexpr int kDeqThreads = 256;      // warps 0-7: dequant + epilogue (two threads per tile row)
constexpr int kCtl = kDeqThreads / 32; // control warp
constexpr int kThreads = kDeqThreads + 32;
// ring stages: as many as shared memory holds next to the table and the A tiles
template <int NP>
__host__ __device__ constexpr int ring_stages() { return NP <= 32 ? 3 : 2; }
constexpr int kWStage = kRows * 128;  // packed bytes per stage: 128 rows x 4 blocks
constexpr int kATile = kRows * 128;   // one dequantised block: 128 rows x 64 weights x 2 bytes
constexpr int kLutBytes5 = 64 * 1024; // 256 entries x 256 B (32 lane copies in the first 128 B)

struct Maps5 {
  CUtensorMap w[kTc5MaxSeg];   // packed weights: [rows, K/2] bytes, boxes 128 rows x 128 B
  CUtensorMap x;               // activations: [M, K] 16-bit, boxes NP tokens x 64 k
};

struct Seg5 {
  const void* absmax;
  int64_t ld_absmax;
  const float* absmax2;
  int64_t gblk_base, gblk_row_stride;
  float offset;
  void* y;
  int64_t ldy;
  int N;
  int tile_end;       // cumulative tile count through this segment
};

struct Args5 {
  int M, K, nstages;  // nstages = K / 256
  int nseg;
  int cs;
  Seg5 seg[kTc5MaxSeg];
  const float* code;
  const float* code2;
  int* err;
};

template <int NP>
__host__ __device__ constexpr uint32_t x_stage_bytes() { return 4u * NP * 128u; }
template <int NP>
constexpr uint32_t smem5_bytes() {
  return kLutBytes5 + ring_stages<NP>() * (kWStage + x_stage_bytes<NP>()) + 2 * kATile + 1024 /* code2 */ +
         128 /* bars */ + 1024 /* alignment slack */;
}

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait: a phase that never completes (only a fault elsewhere could cause it) is counted in the
// error word and the thread carries on, so the launch always ends.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err) {
  for (int i = 0; i < (1 << 22); ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicAdd(err, 1);
  return false;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
// Stage reads and A-tile writes: ordered against the barrier waits and the proxy fence (volatile asm
// with memory clobbers) but free to interleave with the table loads.
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d));
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t local_addr, int rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(local_addr), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];\n" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// Shared-memory matrix descriptor for a K-major operand in the canonical 128-byte-swizzled layout: rows
// of 128 bytes, 8-row groups 1024 bytes apart (stride byte offset), tiles 1024-byte aligned (base
// offset 0), descriptor version 1 (sm_100), layout type 2 = 128-byte swizzle.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}
// Instruction descriptor, kind::f16: fp32 accumulator, A and B of the activation dtype (0 = f16,
// 1 = bf16), both K-major, N = NP, M = 128.
template <typename T, int NP>
__host__ __device__ constexpr uint32_t idesc_f16() {
  return (1u << 4) | ((std::is_same<T, __half>::value ? 0u : 1u) << 7) |
         ((std::is_same<T, __half>::value ? 0u : 1u) << 10) | (static_cast<uint32_t>(NP >> 3) << 17) |
         (static_cast<uint32_t>(kRows >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <typename T> struct Pair;
template <> struct Pair<__half> {
  static __device__ __forceinline__ uint32_t splat(float s) {
    const __half2 h = __float2half2_rn(s);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
};
template <> struct Pair<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t splat(float s) {
    const __nv_bfloat162 h = __float2bfloat162_rn(s);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    const __nv_bfloat162 r =
        __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
};

__device__ __forceinline__ uint32_t lut_pair(const uint8_t* lut, uint32_t word, uint32_t lane4, uint32_t sel) {
  return *reinterpret_cast<const uint32_t*>(lut + __byte_perm(word, lane4, sel));
}

// Tile -> segment and its first row.
__device__ __forceinline__ int seg_of_tile(const Args5& a, int tile, int& row0) {
  int s = 0;
#pragma unroll
  for (int i = 0; i < kTc5MaxSeg - 1; ++i) s += (i + 1 < a.nseg && tile >= a.seg[i].tile_end) ? 1 : 0;
  row0 = (tile - (s ? a.seg[s - 1].tile_end : 0)) * kRows;
  return s;
}

template <typename T, typename OT, bool NESTED, int NP>
__global__ void __launch_bounds__(kThreads, 1) nf4_tc5_kernel(const __grid_constant__ Maps5 maps,
                                                              const __grid_constant__ Args5 a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  constexpr uint32_t kXStage = x_stage_bytes<NP>();
  constexpr int kR = ring_stages<NP>();
  constexpr int kCols = NP <= 32 ? 32 : 64;   // TMEM columns (power of two >= 32)
  pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // 1024-aligned carve-up: table, packed ring, activation ring, A tiles, code2, barriers
  const uint32_t raw_s = smem_u32(smem_raw);
  const uint32_t base = (raw_s + 1023u) & ~1023u;
  uint8_t* const sm = smem_raw + (base - raw_s);
  const uint32_t lut_s = base;
  const uint32_t wring = lut_s + kLutBytes5;
  const uint32_t xring = wring + kR * kWStage;
  const uint32_t abuf = xring + kR * kXStage;
  const uint32_t c2_s = abuf + 2 * kATile;
  const uint32_t bars = c2_s + 1024;
  const uint8_t* lut = sm;
  const float* c2tab = reinterpret_cast<const float*>(sm + (c2_s - base));
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + (bars - base) + 96);
  const uint32_t full = bars, empty = bars + 24, afull = bars + 48, aempty = bars + 64, done = bars + 80;

  // ---- work: tile and this CTA's share of the K stages
  const int cs = a.cs, q = static_cast<int>(blockIdx.x) % cs, tile = static_cast<int>(blockIdx.x) / cs;
  int row0;
  const int sg = seg_of_tile(a, tile, row0);
  const Seg5& S = a.seg[sg];
  const int st0 = q * a.nstages / cs, st1 = (q + 1) * a.nstages / cs, nst = st1 - st0;

  // ---- set-up: barriers, TMEM, tables
  if (tid == kDeqThreads) {
    for (int i = 0; i < kR; ++i) {
      mbar_init(full + 8 * i, 1);
      mbar_init(empty + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(afull + 8 * i, kDeqThreads);
      mbar_init(aempty + 8 * i, 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == kCtl) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  {
    // dequant table: thread e < 256 builds entry e's 32 lane copies (16-byte stores, 4 wavefronts each)
    for (int e = tid; e < 256; e += kThreads) {
      const float hi = __ldg(a.code + (e >> 4)), lo = __ldg(a.code + (e & 15));
      const uint32_t val = Dt<T>::pack2(hi, lo);
      uint4* entry = reinterpret_cast<uint4*>(sm + e * 256);
      const uint4 v4 = make_uint4(val, val, val, val);
#pragma unroll
      for (int i = 0; i < 8; ++i) entry[(i + e) & 7] = v4;
    }
    if (NESTED)
      for (int i = tid; i < 256; i += kThreads) reinterpret_cast<float*>(sm + (c2_s - base))[i] = __ldg(a.code2 + i);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();   // activations and outputs are stream-ordered from here

  if (warp == kCtl) {
    // ---- producer + MMA issuer (one elected thread)
    if (lane == 0 && nst > 0) {
      constexpr uint32_t kIdesc = idesc_f16<T, NP>();
      auto issue = [&](int s) {
        const uint32_t slot = s % kR, bar = full + 8 * slot;
        mbar_expect_tx(bar, kWStage + kXStage);
        tma_load_2d(wring + slot * kWStage, &maps.w[sg], (st0 + s) * 128, row0, bar);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tma_load_2d(xring + slot * kXStage + j * (NP * 128), &maps.x, (st0 + s) * 256 + 64 * j, 0, bar);
      };
      for (int s = 0; s < kR && s < nst; ++s) issue(s);
      const int nkb = 4 * nst;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb >> 2, j = kb & 3;
        if (j == 0) {
          if (s >= 1 && s - 1 + kR < nst) {   // refill the slot the previous stage's MMAs have released
            mbar_wait(empty + 8 * ((s - 1) % kR), static_cast<uint32_t>(((s - 1) / kR) & 1), a.err);
            issue(s - 1 + kR);
          }
          mbar_wait(full + 8 * (s % kR), static_cast<uint32_t>((s / kR) & 1), a.err);
        }
        mbar_wait(afull + 8 * (kb & 1), static_cast<uint32_t>((kb >> 1) & 1), a.err);
        tc_fence_after();
        const uint32_t a_addr = abuf + (kb & 1) * kATile;
        const uint32_t b_addr = xring + (s % kR) * kXStage + j * (NP * 128);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          mma_f16(tmem, sw128_desc(a_addr + 32 * i), sw128_desc(b_addr + 32 * i), kIdesc, (kb | i) != 0 ? 1u : 0u);
        mma_commit(aempty + 8 * (kb & 1));
        if (j == 3) mma_commit(empty + 8 * (s % kR));
      }
      mma_commit(done);
    }
  } else {
    // ---- dequant: thread (h, t) = half h of tile row t (weights 32 h .. 32 h + 31 of every block)
    const int t = tid & (kRows - 1), h = tid >> 7;
    const int64_t row = row0 + t;
    const bool live = row < S.N;
    const uint32_t lane4 = static_cast<uint32_t>(lane) * 4u;
    const uint32_t rsw = static_cast<uint32_t>(t & 7);
    // raw scales of stage s for this row (4 blocks)
    auto load_raw = [&](int s, uint32_t& q4, float& a2, float4& f4) {
      q4 = 0;
      a2 = 0.f;
      f4 = make_float4(0.f, 0.f, 0.f, 0.f);
      if (!live || s >= nst) return;
      const int blk = 4 * (st0 + s);
      if constexpr (NESTED) {
        q4 = __ldg(reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(S.absmax) + row * S.ld_absmax + blk));
        a2 = __ldg(S.absmax2 + ((S.gblk_base + row * S.gblk_row_stride + blk) >> 8));
      } else {
        f4 = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(S.absmax) + row * S.ld_absmax + blk));
      }
    };
    uint32_t q4n;
    float a2n;
    float4 f4n;
    load_raw(0, q4n, a2n, f4n);
    uint32_t sc2[4] = {0, 0, 0, 0};   // block scales of the current stage as paired dtype values
    const int nkb = 4 * nst;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb >> 2, j = kb & 3;
      if (j == 0) {
        float sc[4];
        if constexpr (NESTED) {
#pragma unroll
          for (int i = 0; i < 4; ++i) sc[i] = __fadd_rn(__fmul_rn(c2tab[(q4n >> (8 * i)) & 0xFF], a2n), S.offset);
        } else {
          sc[0] = f4n.x; sc[1] = f4n.y; sc[2] = f4n.z; sc[3] = f4n.w;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) sc2[i] = Pair<T>::splat(sc[i]);
        load_raw(s + 1, q4n, a2n, f4n);
        mbar_wait(full + 8 * (s % kR), static_cast<uint32_t>((s / kR) & 1), a.err);
      }
      if (kb >= 2) mbar_wait(aempty + 8 * (kb & 1), static_cast<uint32_t>(((kb >> 1) - 1) & 1), a.err);
      // packed bytes 16 h .. 16 h + 15 of block j of this row: 16-byte chunk 2j + h of the swizzled
      // 128-byte stage row
      const uint32_t wrow = wring + (s % kR) * kWStage + t * 128;
      const uint4 p0 = lds128(wrow + ((static_cast<uint32_t>(2 * j + h) ^ rsw) << 4));
      const uint32_t pw[4] = {p0.x, p0.y, p0.z, p0.w};
      const uint32_t scl = j == 0 ? sc2[0] : j == 1 ? sc2[1] : j == 2 ? sc2[2] : sc2[3];
      const uint32_t arow = abuf + (kb & 1) * kATile + t * 128;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {   // A chunk c = 4h + cc = weights 8c..8c+7 = packed bytes 4c..4c+3
        const uint32_t w = pw[cc];
        const uint32_t c = static_cast<uint32_t>(4 * h + cc);
        sts128(arow + ((c ^ rsw) << 4),
               Pair<T>::mul(lut_pair(lut, w, lane4, 0x5504u), scl), Pair<T>::mul(lut_pair(lut, w, lane4, 0x5514u), scl),
               Pair<T>::mul(lut_pair(lut, w, lane4, 0x5524u), scl), Pair<T>::mul(lut_pair(lut, w, lane4, 0x5534u), scl));
      }
      fence_proxy_async();   // the generic-proxy stores must be visible to the tensor core's reads
      mbar_arrive(afull + 8 * (kb & 1));
    }

    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (tile rows), columns (tokens)
    // [0, kHalf) for warps 0-3 and [kHalf, NP) for warps 4-7
    if (nst > 0) mbar_wait(done, 0u, a.err);
    __syncwarp();   // the TMEM loads are warp-collective
    tc_fence_after();
    constexpr int kHalf = (NP / 2 + 15) / 16 * 16;
    const int c0 = h ? kHalf : 0, c1 = h ? NP : kHalf;
    float* part = reinterpret_cast<float*>(sm + (xring - base));
#pragma unroll
    for (int c = 0; c < NP; c += 16) {
      if (c < c0 || c >= c1) continue;
      float v[16];
      tmem_ld16(tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + c, v);
      if (cs == 1) {
        if (live) {
          OT* y = static_cast<OT*>(S.y) + row;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (c + i < a.M) y[(c + i) * S.ldy] = Dt<OT>::from_f32(v[i]);
        }
      } else {
        // partial tile into the (now idle) activation ring as [token][row], summed over the cluster
        // by token ranges: CTA q stores tokens [q NP / cs, (q + 1) NP / cs)
#pragma unroll
        for (int i = 0; i < 16; ++i) part[(c + i) * kRows + t] = v[i];
      }
    }
  }
  __syncwarp();
  if (cs > 1) {
    // every thread (the control warp included) takes the cluster barriers
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
    if (tid < kDeqThreads) {
      const int t = tid & (kRows - 1), h = tid >> 7;
      const int64_t row = row0 + t;
      if (row < S.N) {
        OT* y = static_cast<OT*>(S.y) + row;
        const int c0 = q * NP / cs, c1 = (q + 1) * NP / cs;
        for (int c = c0 + h; c < c1 && c < a.M; c += 2) {
          const uint32_t la = xring + static_cast<uint32_t>(c * kRows + t) * 4u;
          float acc = 0.f;
          for (int r = 0; r < cs; ++r) acc += ld_dsmem_f32(la, r);
          y[c * S.ldy] = Dt<OT>::from_f32(acc);
        }
      }
    }
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\nbarrier.cluster.wait.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kCtl) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kCols) : "memory");
  }
}

// ---------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn5() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

bool encode2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
              uint64_t stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  auto fn = encode_fn5();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <typename T, typename OT, bool NESTED, int NP>
int launch5(const Maps5& maps, const Args5& a, int grid, bool pdl, cudaStream_t s) {
  auto kern = nf4_tc5_kernel<T, OT, NESTED, NP>;
  constexpr uint32_t bytes = smem5_bytes<NP>();
  static int configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) !=
        cudaSuccess) {
      cudaGetLastError();
      return kTc5NotApplicable;
    }
    configured[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = bytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, maps, a);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return B2D_ERR_LAUNCH;
  }
  return launch_status();
}

template <typename T, typename OT, bool NESTED>
int launch5_np(const Maps5& maps, const Args5& a, int grid, int np, bool pdl, cudaStream_t s) {
  switch (np) {
    case 16: return launch5<T, OT, NESTED, 16>(maps, a, grid, pdl, s);
    case 32: return launch5<T, OT, NESTED, 32>(maps, a, grid, pdl, s);
    case 48: return launch5<T, OT, NESTED, 48>(maps, a, grid, pdl, s);
    default: return launch5<T, OT, NESTED, 64>(maps, a, grid, pdl, s);
  }
}

template <typename T, typename OT>
int launch5_all(const Maps5& maps, const Args5& a, int grid, int np, bool nested, bool pdl, cudaStream_t s) {
  return nested ? launch5_np<T, OT, true>(maps, a, grid, np, pdl, s)
                : launch5_np<T, OT, false>(maps, a, grid, np, pdl, s);
}

}  // namespace

int nf4_tc5_gemm(const Nf4Tc5Launch& L, cudaStream_t stream) {
  if (L.M < 9 || L.M > 64 || L.K < 256 || L.K % 256 || L.nseg < 1 || L.nseg > kTc5MaxSeg) return kTc5NotApplicable;
  if (!aligned(L.x, 16) || L.ldx % 8 || !L.code_dev) return kTc5NotApplicable;
  if (L.nested && !L.code2) return kTc5NotApplicable;
  DeviceInfo di;
  if (device_info(&di) != B2D_OK) return kTc5NotApplicable;
  Maps5 maps;
  std::memset(&maps, 0, sizeof(maps));
  Args5 a;
  std::memset(&a, 0, sizeof(a));
  a.M = L.M;
  a.K = L.K;
  a.nstages = L.K / 256;
  a.nseg = L.nseg;
  a.code = L.code_dev;
  a.code2 = L.code2;
  a.err = L.err;
  int tiles = 0;
  for (int i = 0; i < L.nseg; ++i) {
    const Nf4Tc5Segment& sg = L.seg[i];
    if (sg.N < 8 || sg.N % 8) return kTc5NotApplicable;
    if (!aligned(sg.packed, 16) || sg.ld_packed % 16 || sg.ld_packed < L.K / 2) return kTc5NotApplicable;
    if (L.nested) {
      if (!aligned(sg.absmax, 4) || sg.ld_absmax % 4 || !sg.absmax2 || sg.gblk_base % 4 || sg.gblk_row_stride % 4)
        return kTc5NotApplicable;
    } else if (!aligned(sg.absmax, 16) || sg.ld_absmax % 4) {
      return kTc5NotApplicable;
    }
    if (!encode2d(&maps.w[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, sg.packed, static_cast<uint64_t>(L.K / 2),
                  static_cast<uint64_t>(sg.N), static_cast<uint64_t>(sg.ld_packed), 128, kRows))
      return kTc5NotApplicable;
    tiles += (sg.N + kRows - 1) / kRows;
    a.seg[i] = Seg5{sg.absmax, sg.ld_absmax, sg.absmax2, sg.gblk_base, sg.gblk_row_stride, sg.offset,
                    sg.y, sg.ldy, sg.N, tiles};
  }
  const int np = (L.M + 15) / 16 * 16;
  if (!encode2d(&maps.x, CU_TENSOR_MAP_DATA_TYPE_UINT16, L.x, static_cast<uint64_t>(L.K), static_cast<uint64_t>(L.M),
                static_cast<uint64_t>(L.ldx) * 2, 64, static_cast<uint32_t>(np)))
    return kTc5NotApplicable;
  // K split: the smallest cluster size that fills the SMs, as long as each CTA keeps at least 4 stages
  int cs = 1;
  while (cs < 4 && tiles * cs * 2 <= di.sm_count && a.nstages / (cs * 2) >= 4) cs *= 2;
  a.cs = cs;
  const int grid = tiles * cs;
  if (L.dtype == B2D_F16)
    return L.y_dtype == B2D_F32 ? launch5_all<__half, float>(maps, a, grid, np, L.nested, L.pdl, stream)
                                : launch5_all<__half, __half>(maps, a, grid, np, L.nested, L.pdl, stream);
  return L.y_dtype == B2D_F32 ? launch5_all<__nv_bfloat16, float>(maps, a, grid, np, L.nested, L.pdl, stream)
                              : launch5_all<__nv_bfloat16, __nv_bfloat16>(maps, a, grid, np, L.nested, L.pdl, stream);
}

}  // namespace b2d
