// Fused NF4 dequant + skinny matmul for decode batches (M <= 8) on sm_100a, weights staged by TMA.
// y[M, N] = x[M, K] @ W[N, K]^T with W in bitsandbytes NF4 (replaces the reference's Triton kernel,
// profiling/kernels/nf4_gemm.py:37-64, and its launcher NF4Weight.matmul, nf4_gemm.py:94-106; same
// storage semantics: row-major packed nibbles, even element in the high nibble, one scale per 64
// weights, optional double-quantised scale code2[q] * absmax2[blk / 256] + offset, fp32 accumulation).
//
// The kernel is bound by two streams: HBM (~0.52 B of weight state per weight) and the shared-memory
// pipe of the dequant-table lookups (one 4-byte lookup per packed byte). Everything else is kept off
// the shared-memory pipe:
//  * Weights: each warp owns a ring of 3 stages of 4 KB in shared memory filled by 2-D tensor copies
//    (cp.async.bulk.tensor: boxes of 8 rows x 128 bytes = 4 blocks of 64 weights, 128-byte swizzle),
//    completed on one mbarrier per stage. No per-lane copy instructions; up to 12 KB per warp in flight.
//  * A unit of work is 32 weight rows (2 MMA row tiles) x 4 blocks; a row chunk is up to 128 rows
//    (8 tiles, whose accumulators stay in registers). Fragment reads are two 4-byte words per row and
//    block, conflict-free under the 128-byte swizzle.
//  * Activations: every warp owns a fixed slice of at most 8 blocks of K for the whole launch, so the
//    activations of its slice (8 tokens x 512 k) are loaded into registers once, after the dependency
//    wait, and reused for every row tile.
//  * Dequant: a 256-entry table maps a packed byte to the pair (code[hi], code[lo]) in the activation
//    dtype = one tensor-core A-fragment register; entry e, lane l at byte 256 e + 4 l (one byte permute
//    forms the address, every lookup hits 32 distinct banks). The other half of each 256-byte row holds
//    32 lane copies of the double-quant table code2, so scale decoding is conflict-free too.
//  * The block scale is factored out of the dot product: four m16n8k16 MMAs per block accumulate
//    sum_k x_k * code[n_k] from zero and one fp32 FMA per output applies the scale. The MMA reduction
//    axis is permuted so that a lane's two weight words per row and its two 16-byte activation loads
//    cover the same k values: lane (g, t) owns k in [8t, 8t+8) and [32+8t, 32+8t+8) of each block.
//  * Partition: clusters of 1, 2 or 4 CTAs (chosen per shape by the host); a cluster owns a contiguous
//    range of 8-row units (balanced to one unit), its CTAs split K evenly, and the warps of a CTA split
//    the CTA's K range evenly while all working on the same rows. A CTA's warps reduce their partial
//    products through shared memory at the end of every row chunk; the CTAs of a cluster reduce theirs
//    through distributed shared memory at the end, in rank order, so results are deterministic.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "nf4_tma.cuh"

namespace b2d {
namespace {

constexpr int kRing = 3;                 // stages per warp
constexpr int kTmaLutBytes = 64 * 1024;  // 256 entries x 256 B: dequant pairs (bytes 0..127) + code2 (128..255)
constexpr int kMaxChunks = 4;            // row chunks per cluster whose partials are kept for the cluster sum
constexpr int kEpiStore = 0, kEpiPair = 1, kEpiAllReduce = 2;

struct TmaMaps {
  CUtensorMap m[kTmaMaxSeg];    // boxes of one full 32-row unit (silu_mul: 16 rows of each segment) x 128 B
  CUtensorMap m8[kTmaMaxSeg];   // boxes of 8 rows x 128 B (partial units, units straddling two segments)
};

struct TSeg {
  const void* absmax;
  int64_t ld_absmax;
  const float* absmax2;
  int64_t gblk_base, gblk_row_stride;
  float offset;
  void* y;
  int64_t ldy;
  int row_begin;      // first row of this segment in the launch's row space (independent mode)
};

struct TArgs {
  const void* x;
  int64_t ldx;
  int M, K, nb;       // nb = K / 64
  int nseg;
  int static_w;
  int ru_total;       // row units: 8-row units (independent / all-reduce) or 8 output rows (silu_mul)
  int seg_end_ru[kTmaMaxSeg];
  int N;              // all-reduce: output rows (words per token pair)
  float code_v[16];
  int code_by_value;
  const float* code_dev;
  const float* code2;
  TSeg seg[kTmaMaxSeg];
  ArPeers are;
  int* err;
};

constexpr int kStage = 4096;            // one unit: 32 rows x 128 bytes (4 blocks)
constexpr int kSbStride = 20;           // floats per fragment row g in the scale buffer (bank spread)
constexpr int kSbFloats = 8 * kSbStride;

template <int NW, int MAXT>
constexpr size_t tma_smem_bytes() {
  return kTmaLutBytes + static_cast<size_t>(NW) * kRing * kStage          // rings
         + static_cast<size_t>(NW) * MAXT * 512                          // per-warp tile partials
         + static_cast<size_t>(kMaxChunks) * MAXT * 512                  // CTA chunk partials (cluster sum)
         + static_cast<size_t>(NW) * 2 * kSbFloats * 4                   // decoded scales, double-buffered
         + static_cast<size_t>(NW) * kRing * 8 + 64;                     // mbarriers
}

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait: a stage that never completes (which only a fault elsewhere could cause) is counted in
// the error word and the warp carries on with whatever the stage holds, so the launch always ends.
__device__ __forceinline__ void mbar_wait(uint32_t bar, uint32_t parity, int* err) {
  for (int i = 0; i < (1 << 22); ++i)
    if (mbar_try_wait(bar, parity)) return;
  if (err && (threadIdx.x & 31) == 0) atomicAdd(err, 1);
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];\n" ::"l"(p));
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
// Activations are the previous kernel's output: read with coherent loads in volatile asm so that they
// cannot be scheduled above the dependency wait.
__device__ __forceinline__ uint4 ld_act_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ int seg_of_ru(const TArgs& a, int ru) {
  int s = 0;
#pragma unroll
  for (int i = 0; i < kTmaMaxSeg - 1; ++i) s += (i + 1 < a.nseg && ru >= a.seg_end_ru[i]) ? 1 : 0;
  return s;
}

// Scale state of one lane for one 32-row sub-chunk: the raw scales of its row (row 32 I + lane of the
// chunk) over the warp's blocks.
template <bool NESTED> struct ScaleRow;
template <> struct ScaleRow<true> {
  uint2 raw;           // byte j = code2 index of block wb0 + j
  float a2lo, a2hi, off;
  int jsplit;          // blocks j < jsplit use a2lo, the rest a2hi (a 256-block group boundary)
};
template <> struct ScaleRow<false> {
  float f[8];
};

// Segment and segment-local row of chunk row r (r = 16 t + 8 h + g: tile t, half h, fragment row g).
template <int EPI>
__device__ __forceinline__ bool row_of(const TArgs& a, int rb, int nru, int r, int& s, int64_t& row) {
  if (EPI == kEpiPair) {
    const int t = r >> 4;
    s = (r >> 3) & 1;
    row = 8ll * (rb + t) + (r & 7);
    return t < nru;
  }
  const int hh = r >> 3;
  if (hh >= nru) return false;
  s = seg_of_ru(a, rb + hh);
  row = 8ll * (rb + hh) + (r & 7) - a.seg[s].row_begin;
  return true;
}

// Rows past the chunk get zero scales (their outputs are never stored).
template <bool NESTED, int EPI>
__device__ __forceinline__ void load_scale_row(ScaleRow<NESTED>& sr, const TArgs& a, int rb, int nru, int r, int wb0,
                                               int nbw) {
  int s = 0;
  int64_t row = 0;
  const bool ok = nbw > 0 && row_of<EPI>(a, rb, nru, r, s, row);
  if constexpr (NESTED) {
    sr.raw = make_uint2(0, 0);
    sr.a2lo = sr.a2hi = sr.off = 0.f;
    sr.jsplit = 8;
    if (!ok) return;
    const TSeg& sg = a.seg[s];
    // the 4-byte words covering bytes [wb0, wb0 + nbw) of the row (the host checks 4-byte alignment of
    // the table and its stride, so no word leaves the row's own 4-byte-rounded span)
    const uint8_t* p = static_cast<const uint8_t*>(sg.absmax) + row * sg.ld_absmax + wb0;
    const uintptr_t A = reinterpret_cast<uintptr_t>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(A & ~uintptr_t(3));
    const int sh = static_cast<int>(A & 3);
    const int last = (sh + nbw - 1) >> 2;
    const uint32_t w0 = __ldg(w);
    const uint32_t w1 = last >= 1 ? __ldg(w + 1) : 0u;
    const uint32_t w2 = last >= 2 ? __ldg(w + 2) : 0u;
    sr.raw.x = __funnelshift_r(w0, w1, 8 * sh);
    sr.raw.y = __funnelshift_r(w1, w2, 8 * sh);
    const int64_t gb = sg.gblk_base + row * sg.gblk_row_stride + wb0;
    const int64_t i0 = gb >> 8;
    const int js = 256 - static_cast<int>(gb & 255);
    sr.jsplit = js;
    sr.a2lo = __ldg(sg.absmax2 + i0);
    sr.a2hi = js < nbw ? __ldg(sg.absmax2 + i0 + 1) : sr.a2lo;
    sr.off = sg.offset;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) sr.f[j] = 0.f;
    if (!ok) return;
    const TSeg& sg = a.seg[s];
    const float* p = static_cast<const float*>(sg.absmax) + row * sg.ld_absmax + wb0;
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
      for (int q = 0; q < 2; ++q)
        if (4 * q + 4 <= nbw) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(p) + q);
          sr.f[4 * q] = v.x; sr.f[4 * q + 1] = v.y; sr.f[4 * q + 2] = v.z; sr.f[4 * q + 3] = v.w;
        } else {
#pragma unroll
          for (int j = 4 * q; j < 4 * q + 4; ++j)
            if (j < nbw) sr.f[j] = __ldg(p + j);
        }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < nbw) sr.f[j] = __ldg(p + j);
    }
  }
}

// Decodes the scales of block group BG of this lane's row into the warp's scale buffer, in fragment
// order: sb[g * stride + 4 (2 tt + h) + jj] = scale of block 4 BG + jj of the sub-chunk's row 16 tt + 8 h + g.
template <bool NESTED, int BG>
__device__ __forceinline__ void decode_scales_unit(const ScaleRow<NESTED>& sr, float* sb, const uint8_t* lut,
                                                   uint32_t lane_c2, int lane) {
  float v[4];
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    if constexpr (NESTED) {
      const uint32_t qw = BG == 0 ? sr.raw.x : sr.raw.y;
      const float c2 = *reinterpret_cast<const float*>(lut + __byte_perm(qw, lane_c2, 0x5504u + 0x10u * jj));
      const float a2 = 4 * BG + jj < sr.jsplit ? sr.a2lo : sr.a2hi;
      v[jj] = __fadd_rn(__fmul_rn(c2, a2), sr.off);
    } else {
      v[jj] = sr.f[4 * BG + jj];
    }
  }
  *reinterpret_cast<float4*>(sb + (lane & 7) * kSbStride + 4 * (lane >> 3)) = make_float4(v[0], v[1], v[2], v[3]);
}

__device__ __forceinline__ uint32_t lut_at(const uint8_t* lut, uint32_t word, uint32_t lane4, uint32_t sel) {
  return *reinterpret_cast<const uint32_t*>(lut + __byte_perm(word, lane4, sel));
}

// One unit: the stage's 2 row tiles x 4 blocks, accumulated into acc[2]. No guards: rows the copy did not
// fill hold stale (finite: every byte is a valid table index) values whose outputs are never stored, and
// blocks past the warp's slice meet zero activations and zero scales. roff[tt][h] = byte offset of row
// 16 tt + 8 h + g; cofs[j] = the lane's two word offsets of block j under the 128-byte swizzle.
template <typename T, int BG, uint32_t HALF>
__device__ __forceinline__ void compute_unit(const uint8_t* stage, const uint32_t (&roff)[2],
                                             const uint32_t (&cofs)[4][2], const uint4 (&xr)[8][2], const float* sb,
                                             int g, float (&acc)[2][4], const uint8_t* lut, uint32_t lane4) {
#pragma unroll
  for (int tt = 0; tt < 2; ++tt) {
    const uint8_t* r0 = stage + roff[tt];   // row g of the tile; row g + 8 is HALF bytes further
    const float4 s0 = *reinterpret_cast<const float4*>(sb + g * kSbStride + 4 * (2 * tt));
    const float4 s1 = *reinterpret_cast<const float4*>(sb + g * kSbStride + 4 * (2 * tt + 1));
    const float sc0[4] = {s0.x, s0.y, s0.z, s0.w}, sc1[4] = {s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const uint32_t lo0 = lds32(r0 + cofs[jj][0]), hi0 = lds32(r0 + cofs[jj][1]);
      const uint32_t lo1 = lds32(r0 + HALF + cofs[jj][0]), hi1 = lds32(r0 + HALF + cofs[jj][1]);
      const uint4& xa = xr[4 * BG + jj][0];
      const uint4& xb = xr[4 * BG + jj][1];
      float c[4];
      Mma<T>::run0(c, lut_at(lut, lo0, lane4, 0x5504u), lut_at(lut, lo1, lane4, 0x5504u),
                   lut_at(lut, lo0, lane4, 0x5514u), lut_at(lut, lo1, lane4, 0x5514u), xa.x, xa.y);
      Mma<T>::run(c, lut_at(lut, lo0, lane4, 0x5524u), lut_at(lut, lo1, lane4, 0x5524u),
                  lut_at(lut, lo0, lane4, 0x5534u), lut_at(lut, lo1, lane4, 0x5534u), xa.z, xa.w);
      Mma<T>::run(c, lut_at(lut, hi0, lane4, 0x5504u), lut_at(lut, hi1, lane4, 0x5504u),
                  lut_at(lut, hi0, lane4, 0x5514u), lut_at(lut, hi1, lane4, 0x5514u), xb.x, xb.y);
      Mma<T>::run(c, lut_at(lut, hi0, lane4, 0x5524u), lut_at(lut, hi1, lane4, 0x5524u),
                  lut_at(lut, hi0, lane4, 0x5534u), lut_at(lut, hi1, lane4, 0x5534u), xb.z, xb.w);
      acc[tt][0] = fmaf(sc0[jj], c[0], acc[tt][0]);
      acc[tt][1] = fmaf(sc0[jj], c[1], acc[tt][1]);
      acc[tt][2] = fmaf(sc1[jj], c[2], acc[tt][2]);
      acc[tt][3] = fmaf(sc1[jj], c[3], acc[tt][3]);
    }
  }
}

// SwiGLU in the model dtype, as a Mistral MLP computes it: act_fn(gate_proj(x)) * up_proj(x) with every
// intermediate rounded to OT.
template <typename OT>
__device__ __forceinline__ OT swiglu(float gate, float up) {
  const float gq = Dt<OT>::to_f32(Dt<OT>::from_f32(gate));
  const float sq = Dt<OT>::to_f32(Dt<OT>::from_f32(gq / (1.0f + expf(-gq))));
  return Dt<OT>::from_f32(sq * Dt<OT>::to_f32(Dt<OT>::from_f32(up)));
}

// Stores tile t of the chunk starting at row unit rb (nru units) from fragment order: v = (row g, token
// 2tq), (row g, 2tq+1), (row g+8, 2tq), (row g+8, 2tq+1).
template <typename OT, int EPI>
__device__ __forceinline__ void store_tile(const TArgs& a, int rb, int nru, int t, float4 v, int g, int tq,
                                           uint32_t epoch) {
  const int t0 = 2 * tq;
  if constexpr (EPI == kEpiPair) {
    OT* y = static_cast<OT*>(a.seg[0].y);
    const int64_t orow = 8ll * (rb + t) + g;
    if (t0 < a.M) y[t0 * a.seg[0].ldy + orow] = swiglu<OT>(v.x, v.z);
    if (t0 + 1 < a.M) y[(t0 + 1) * a.seg[0].ldy + orow] = swiglu<OT>(v.y, v.w);
    return;
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int hh = 2 * t + h;
    if (hh >= nru) break;
    const float lo = h ? v.z : v.x, hi = h ? v.w : v.y;
    const int64_t grow = 8ll * (rb + hh) + g;
    if constexpr (EPI == kEpiAllReduce) {
      if constexpr (!std::is_same<OT, float>::value) {
        if (t0 < a.M) {
          const uint64_t word = (static_cast<uint64_t>(epoch) << 32) | Dt<OT>::pack2(lo, hi);
          const int64_t w = static_cast<int64_t>(tq) * a.N + grow;
          for (int p = 0; p < a.are.world; ++p) st_word(ar_slot(a.are, p, a.are.rank, epoch) + w, word);
        }
      }
    } else {
      const int s = seg_of_ru(a, rb + hh);
      OT* y = static_cast<OT*>(a.seg[s].y);
      const int64_t row = grow - a.seg[s].row_begin;
      const int64_t ldy = a.seg[s].ldy;
      if (t0 < a.M) y[t0 * ldy + row] = Dt<OT>::from_f32(lo);
      if (t0 + 1 < a.M) y[(t0 + 1) * ldy + row] = Dt<OT>::from_f32(hi);
    }
  }
}

template <typename T, typename OT, bool NESTED, int EPI, int NW, int MAXT>
__global__ void __launch_bounds__(NW * 32, 1) nf4_tma_kernel(const __grid_constant__ TmaMaps maps,
                                                             const __grid_constant__ TArgs a) {
  constexpr int RPC = EPI == kEpiPair ? MAXT : 2 * MAXT;   // row units per chunk
  constexpr int RPS = EPI == kEpiPair ? 2 : 4;             // row units per 32-row sub-chunk
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* lut = smem;
  uint8_t* rings = smem + kTmaLutBytes;
  float* slots = reinterpret_cast<float*>(rings + NW * kRing * kStage);           // [NW][MAXT][32 lanes][4]
  float* cpart = slots + NW * MAXT * 128;                                         // [kMaxChunks][MAXT][32][4]
  float* sbufs = cpart + kMaxChunks * MAXT * 128;                                 // [NW][2][kSbFloats]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sbufs + NW * 2 * kSbFloats);       // [NW][kRing]

  pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // The fragment reads assume the 128-byte swizzle pattern relative to 1024-byte aligned boxes: a launch
  // whose shared memory is not 1024-byte aligned records an error and does nothing (the same for every
  // CTA, so no cluster barrier is left waiting).
  if ((smem_u32(smem) & 1023u) != 0) {
    if (tid == 0 && a.err) atomicAdd(a.err, 1 << 16);
    return;
  }
  const int g = lane >> 2, tq = lane & 3;
  const uint32_t lane4 = static_cast<uint32_t>(lane) * 4u;
  const uint32_t lane_c2 = 128u + lane4;

  // ---- partition (32-bit math; the host keeps ru_total * clusters and nb * cs below 2^31)
  const int cs = cluster_size(), q = cluster_rank(), cl = cluster_index(), ncl = cluster_count();
  const int ru0 = cl * a.ru_total / ncl, ru1 = (cl + 1) * a.ru_total / ncl;
  const int nchunks = (ru1 - ru0 + RPC - 1) / RPC;
  const int kb0 = q * a.nb / cs, kb1 = (q + 1) * a.nb / cs;
  const int wb0 = kb0 + warp * (kb1 - kb0) / NW, wb1 = kb0 + (warp + 1) * (kb1 - kb0) / NW;
  const int nbw = wb1 - wb0;          // <= 8 (host)
  const int ngroups = (nbw + 3) / 4;  // 4-block groups of this warp's slice

  uint8_t* ring = rings + warp * kRing * kStage;
  const uint32_t ring_s = smem_u32(ring);
  const uint32_t bar_s = smem_u32(bars + warp * kRing);
  float* sbw = sbufs + warp * 2 * kSbFloats;
  if (lane == 0) {
    for (int s = 0; s < kRing; ++s) mbar_init(bar_s + 8 * s, 1);
    fence_mbar_init();
  }
  __syncwarp();

  // Copies the boxes of unit (chunk ic, sub-chunk ii, block group ig) into stage st.
  auto unit_boxes = [&](int ic, int ii, int ig, uint32_t st, uint32_t bar) {
    const int rb = ru0 + ic * RPC, nru = min(RPC, ru1 - rb);
    const int u0 = ii * RPS, u1 = min(u0 + RPS, nru);
    mbar_expect_tx(bar, static_cast<uint32_t>(u1 - u0) * (EPI == kEpiPair ? 2048u : 1024u));
    const int xk = (wb0 + 4 * ig) * 32;
    auto box = [&](uint32_t dst, const CUtensorMap* m, int y) { tma_load_2d(dst, m, xk, y, bar); };
    // silu_mul layout: gate rows of the unit's two tiles in the first 2 KB, up rows in the second
    if (EPI == kEpiPair) {
      if (u1 - u0 == RPS) {
        box(st, &maps.m[0], 8 * (rb + u0));
        box(st + 2048, &maps.m[1], 8 * (rb + u0));
      } else {
        for (int r = u0; r < u1; ++r) {
          box(st + (r - u0) * 1024, &maps.m8[0], 8 * (rb + r));
          box(st + 2048 + (r - u0) * 1024, &maps.m8[1], 8 * (rb + r));
        }
      }
    } else {
      const int s0 = seg_of_ru(a, rb + u0);
      if (u1 - u0 == RPS && seg_of_ru(a, rb + u1 - 1) == s0) {
        box(st, &maps.m[s0], 8 * (rb + u0) - a.seg[s0].row_begin);
      } else {
        for (int r = u0; r < u1; ++r) {
          const int s = seg_of_ru(a, rb + r);
          box(st + (r - u0) * 1024, &maps.m8[s], 8 * (rb + r) - a.seg[s].row_begin);
        }
      }
    }
  };
  // Issue cursor (lane 0): the next unit to copy, in consumption order chunk -> sub-chunk -> block group.
  int ic = 0, ii = 0, ig = 0, iu = 0;
  auto step_cursor = [&](int& c, int& i, int& g2) {
    const int nru = min(RPC, ru1 - (ru0 + c * RPC));
    if (++g2 == ngroups) {
      g2 = 0;
      if (++i == (nru + RPS - 1) / RPS) { i = 0; ++c; }
    }
  };
  auto issue_next = [&]() {   // lane 0
    if (ic >= nchunks || ngroups == 0) return;
    unit_boxes(ic, ii, ig, ring_s + (iu % kRing) * kStage, bar_s + 8 * (iu % kRing));
    ++iu;
    step_cursor(ic, ii, ig);
  };

  // Weights and scales start streaming before the table is built: at once when they do not depend on
  // the preceding kernel (static weights), else right after the dependency wait.
  if (!a.static_w) pdl_wait();
  // Scale row of the lane for sub-chunk I of chunk c (row 32 I + lane of the chunk).
  auto load_sub = [&](ScaleRow<NESTED>& dst, int c, int I) {
    if (c < nchunks) {
      const int rb = ru0 + c * RPC;
      load_scale_row<NESTED, EPI>(dst, a, rb, min(RPC, ru1 - rb), 32 * I + lane, wb0, nbw);
    }
  };
  ScaleRow<NESTED> sr;
  if (lane == 0)
    for (int k = 0; k < kRing; ++k) issue_next();
  // The scale bytes and group scales of every row of the cluster's range over this warp's blocks go to
  // L1 now (a few KB per CTA), so the per-sub-chunk loads below hit L1 instead of waiting on L2 / HBM.
  if (nbw > 0) {
    for (int r = lane; r < (ru1 - ru0) * (EPI == kEpiPair ? 16 : 8); r += 32) {
      int s = 0;
      int64_t row = 0;
      const int c = r / (16 * (EPI == kEpiPair ? MAXT : MAXT)), rr = r - c * 16 * MAXT;
      if (!row_of<EPI>(a, ru0 + c * RPC, min(RPC, ru1 - (ru0 + c * RPC)), rr, s, row)) continue;
      const TSeg& sg = a.seg[s];
      const uint8_t* p = static_cast<const uint8_t*>(sg.absmax) + (row * sg.ld_absmax + wb0) * (NESTED ? 1 : 4);
      prefetch_l1(p);
      prefetch_l1(p + (NESTED ? nbw - 1 : 4 * nbw - 4));
      if (NESTED) prefetch_l1(sg.absmax2 + ((sg.gblk_base + row * sg.gblk_row_stride + wb0) >> 8));
    }
  }

  // ---- dequant table + code2 lane copies (lane-rotated stores: 32 distinct banks per instruction)
  {
    const float my_code = a.code_by_value ? a.code_v[lane & 15] : __ldg(a.code_dev + (lane & 15));
    for (int ew = warp; ew < 8; ew += NW) {
      const int e = ew * 32 + lane;
      const float hi = __shfl_sync(0xffffffffu, my_code, (e >> 4) & 15);
      const float lo = __shfl_sync(0xffffffffu, my_code, e & 15);
      const uint32_t val = Dt<T>::pack2(hi, lo);
      uint32_t* entry = reinterpret_cast<uint32_t*>(lut + e * 256);
#pragma unroll
      for (int i = 0; i < 32; ++i) entry[(i + lane) & 31] = val;
      if (NESTED) {
        const float c2 = __ldg(a.code2 + e);
        float* e2 = reinterpret_cast<float*>(lut + e * 256 + 128);
#pragma unroll
        for (int i = 0; i < 32; ++i) e2[(i + lane) & 31] = c2;
      }
    }
  }
  __syncthreads();
  pdl_wait();   // activations and outputs are stream-ordered from here
  const uint32_t epoch = EPI == kEpiAllReduce ? ar_epoch(a.are) : 0u;

  // ---- this warp's activations: 8 tokens x its blocks, lane (g, tq) -> token g, k 8tq.. and 32+8tq..;
  // blocks past the slice are zero
  uint4 xr[8][2];
  {
    const int tok = g < a.M ? g : 0;   // rows past M read token 0; their outputs are never stored
    const T* xp = static_cast<const T*>(a.x) + static_cast<int64_t>(tok) * a.ldx + wb0 * 64 + 8 * tq;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j < nbw) {
        xr[j][0] = ld_act_u4(xp + j * 64);
        xr[j][1] = ld_act_u4(xp + j * 64 + 32);
      } else {
        xr[j][0] = xr[j][1] = make_uint4(0, 0, 0, 0);
      }
    }
  }
  // per-lane fragment offsets: rows g (+8 = +1 KB) of the unit's two tiles, and the two words of each
  // block (128-byte swizzle: 16-byte chunk c of box row r sits at chunk c ^ r, with r == g)
  // row g of tile tt: plain units hold rows 16 tt + 8 h + g in order; silu_mul units hold the gate rows
  // (h = 0) of both tiles first and the up rows (h = 1) 2 KB further
  const uint32_t roff[2] = {static_cast<uint32_t>(g) * 128u,
                            static_cast<uint32_t>((EPI == kEpiPair ? 8 : 16) + g) * 128u};
  constexpr uint32_t kHalfOff = EPI == kEpiPair ? 2048u : 1024u;   // from row g to row g + 8 of a tile
  uint32_t cofs[4][2];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    cofs[j][0] = ((static_cast<uint32_t>(2 * j) ^ g) << 4) + 4u * tq;
    cofs[j][1] = ((static_cast<uint32_t>(2 * j + 1) ^ g) << 4) + 4u * tq;
  }

  int u = 0;   // units consumed (stage u % kRing, phase (u / kRing) & 1)
  for (int c = 0; c < nchunks; ++c) {
    const int rb = ru0 + c * RPC, nru = min(RPC, ru1 - rb);
    const int nt = EPI == kEpiPair ? nru : (nru + 1) / 2;
    const int nsub = (nru + RPS - 1) / RPS;
    for (int I = 0; I < nsub; ++I) {
      load_sub(sr, c, I);   // L1 hits (prefetched at the start)
      float acc[2][4] = {};
#define B2D_TMA_UNIT(BG)                                                                                      \
      if (BG < ngroups) {                                                                                     \
        float* sb = sbw + BG * kSbFloats;                                                                     \
        decode_scales_unit<NESTED, BG>(sr, sb, lut, lane_c2, lane);                                           \
        __syncwarp();                                                                                         \
        const uint32_t st = u % kRing;                                                                        \
        mbar_wait(bar_s + 8 * st, static_cast<uint32_t>((u / kRing) & 1), a.err);                             \
        compute_unit<T, BG, kHalfOff>(ring + st * kStage, roff, cofs, xr, sb, g, acc, lut, lane4);            \
        __syncwarp();                                                                                         \
        if (lane == 0) issue_next();   /* the stage's bytes were consumed by the MMAs above */             \
        ++u;                                                                                                  \
      }
      B2D_TMA_UNIT(0) B2D_TMA_UNIT(1)
#undef B2D_TMA_UNIT
#pragma unroll
      for (int tt = 0; tt < 2; ++tt)
        *reinterpret_cast<float4*>(slots + ((warp * MAXT + 2 * I + tt) * 32 + lane) * 4) =
            make_float4(acc[tt][0], acc[tt][1], acc[tt][2], acc[tt][3]);
    }
    // ---- the CTA's sum over its warps (warp order), tile t by warp t % NW
    named_bar(1, NW * 32);
    for (int t = warp; t < nt; t += NW) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int w = 0; w < NW; ++w) {
        const float4 p = *reinterpret_cast<const float4*>(slots + ((w * MAXT + t) * 32 + lane) * 4);
        v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
      }
      if (cs == 1) store_tile<OT, EPI>(a, rb, nru, t, v, g, tq, epoch);
      else *reinterpret_cast<float4*>(cpart + ((c * MAXT + t) * 32 + lane) * 4) = v;
    }
    named_bar(1, NW * 32);
  }
  if (cs == 1) return;
  // ---- the cluster's sum over its CTAs (rank order); chunk c is stored by CTA c % cs
  cluster_sync();
  for (int c = q; c < nchunks; c += cs) {
    const int rb = ru0 + c * RPC, nru = min(RPC, ru1 - rb);
    const int nt = EPI == kEpiPair ? nru : (nru + 1) / 2;
    for (int t = warp; t < nt; t += NW) {
      const uint32_t la = smem_u32(cpart + ((c * MAXT + t) * 32 + lane) * 4);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < cs; ++r) {
        const float4 p = ld_dsmem_f4(la, r);
        v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
      }
      store_tile<OT, EPI>(a, rb, nru, t, v, g, tq, epoch);
    }
  }
  // keeps every CTA's partials alive until the owners have read them (their values are consumed)
  cluster_sync_relaxed();
}

// ---------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// Packed bytes of one weight (segment) as a 2-D uint8 tensor [rows, K/2] with row stride ld_packed; boxes
// of box_rows rows x 128 bytes (four 64-weight blocks), 128-byte swizzle.
bool encode_packed(CUtensorMap* m, const uint8_t* packed, int64_t ld_packed, int rows, int K, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K / 2), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_packed)};
  cuuint32_t box[2] = {128, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(packed), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct TmaConfig {
  int nw, maxt, cs, ncl;
};

template <typename T, typename OT, bool NESTED, int EPI, int NW, int MAXT>
struct TmaKernel {
  static constexpr size_t kSmem = tma_smem_bytes<NW, MAXT>();
  static void* fn() { return reinterpret_cast<void*>(nf4_tma_kernel<T, OT, NESTED, EPI, NW, MAXT>); }
  // Max active clusters of size 1, 2, 4 for this instantiation on the current device (queried once).
  static const int* max_clusters(int dev) {
    static int table[64][3];
    static std::once_flag once[64];
    std::call_once(once[dev], [&] {
      auto kern = nf4_tma_kernel<T, OT, NESTED, EPI, NW, MAXT>;
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmem)) !=
          cudaSuccess) {
        cudaGetLastError();
        for (int i = 0; i < 3; ++i) table[dev][i] = -1;
        return;
      }
      DeviceInfo di;
      device_info(&di);
      for (int i = 0; i < 3; ++i) {
        const int cs = 1 << i;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(cs * (di.sm_count / cs));
        cfg.blockDim = dim3(NW * 32);
        cfg.dynamicSmemBytes = kSmem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = cs;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int m = 0;
        if (cudaOccupancyMaxActiveClusters(&m, kern, &cfg) != cudaSuccess || m <= 0) {
          cudaGetLastError();
          m = i == 0 ? di.sm_count : -1;
        }
        table[dev][i] = m;
      }
    });
    return table[dev];
  }
  static int launch(const TmaMaps& maps, const TArgs& a, const TmaConfig& c, bool pdl, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c.cs * c.ncl);
    cfg.blockDim = dim3(NW * 32);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = c.cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, nf4_tma_kernel<T, OT, NESTED, EPI, NW, MAXT>, maps, a);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return B2D_ERR_LAUNCH;
    }
    return launch_status();
  }
};

// Picks the cluster size: every CTA's K range split over NW warps must be at most 8 blocks (the
// activations stay in registers), and among those the configuration with the least work on the busiest
// CTA (row units per cluster x blocks per CTA) wins; ties go to the smaller cluster.
template <class K>
bool choose(const TArgs& a, int dev, TmaConfig* out, int nw, int maxt, int rpc) {
  const int* mc = K::max_clusters(dev);
  int64_t best = -1;
  for (int i = 0; i < 3; ++i) {
    const int cs = 1 << i;
    if (mc[i] <= 0) continue;
    const int kc = (a.nb + cs - 1) / cs;
    if ((kc + nw - 1) / nw > 8) continue;
    const int ncl = mc[i] < a.ru_total ? mc[i] : a.ru_total;
    const int per = (a.ru_total + ncl - 1) / ncl;
    if (cs > 1 && (per + rpc - 1) / rpc > kMaxChunks) continue;
    const int64_t work = static_cast<int64_t>(per) * kc;
    if (best < 0 || work < best) {
      best = work;
      *out = TmaConfig{nw, maxt, cs, ncl};
    }
  }
  return best >= 0;
}

template <typename T, typename OT, bool NESTED, int EPI>
int dispatch(const TmaMaps& maps, const TArgs& a, int dev, bool pdl, cudaStream_t s) {
  using K8 = TmaKernel<T, OT, NESTED, EPI, 8, 8>;
  TmaConfig c;
  if (!choose<K8>(a, dev, &c, 8, 8, EPI == kEpiPair ? 8 : 16)) return kTmaNotApplicable;
  return K8::launch(maps, a, c, pdl, s);
}

template <typename T, typename OT>
int dispatch_mode(const Nf4TmaLaunch& L, const TmaMaps& maps, const TArgs& a, int dev, cudaStream_t s) {
  if (L.mode == kTmaIndependent)
    return L.nested ? dispatch<T, OT, true, kEpiStore>(maps, a, dev, L.pdl, s)
                    : dispatch<T, OT, false, kEpiStore>(maps, a, dev, L.pdl, s);
  if constexpr (std::is_same<T, OT>::value) {
    if (L.mode == kTmaSiluMul)
      return L.nested ? dispatch<T, OT, true, kEpiPair>(maps, a, dev, L.pdl, s)
                      : dispatch<T, OT, false, kEpiPair>(maps, a, dev, L.pdl, s);
    if (L.mode == kTmaAllReduce)
      return L.nested ? dispatch<T, OT, true, kEpiAllReduce>(maps, a, dev, L.pdl, s)
                      : dispatch<T, OT, false, kEpiAllReduce>(maps, a, dev, L.pdl, s);
  }
  return kTmaNotApplicable;
}

}  // namespace

int nf4_tma_gemm(const Nf4TmaLaunch& L, cudaStream_t stream) {
  if (L.M < 1 || L.M > 8 || L.K < 64 || L.K % 64 || L.nseg < 1 || L.nseg > kTmaMaxSeg) return kTmaNotApplicable;
  if (L.mode == kTmaSiluMul && (L.nseg != 2 || L.seg[0].N != L.seg[1].N)) return kTmaNotApplicable;
  if (L.mode == kTmaAllReduce && L.nseg != 1) return kTmaNotApplicable;
  if (!aligned(L.x, 16) || L.ldx % 8) return kTmaNotApplicable;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kTmaNotApplicable;
  TmaMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  TArgs a;
  std::memset(&a, 0, sizeof(a));
  a.x = L.x;
  a.ldx = L.ldx;
  a.M = L.M;
  a.K = L.K;
  a.nb = L.K / 64;
  a.nseg = L.nseg;
  a.static_w = L.static_w ? 1 : 0;
  a.err = L.err;
  a.code_dev = L.code_dev;
  if (L.code_host) {
    a.code_by_value = 1;
    for (int i = 0; i < 16; ++i) a.code_v[i] = L.code_host[i];
  }
  a.code2 = L.seg[0].code2;
  int rows_total = 0;
  for (int i = 0; i < L.nseg; ++i) {
    const Nf4TmaSegment& sg = L.seg[i];
    if (sg.N < 8 || sg.N % 8) return kTmaNotApplicable;
    if (!aligned(sg.packed, 16) || sg.ld_packed % 16 || sg.ld_packed < L.K / 2) return kTmaNotApplicable;
    if (L.nested) {
      if (!aligned(sg.absmax, 4) || sg.ld_absmax % 4 || sg.code2 != L.seg[0].code2 || !sg.code2 || !sg.absmax2)
        return kTmaNotApplicable;
    } else if (!aligned(sg.absmax, 4)) {
      return kTmaNotApplicable;
    }
    if (!encode_packed(&maps.m[i], sg.packed, sg.ld_packed, sg.N, L.K, L.mode == kTmaSiluMul ? 16 : 32) ||
        !encode_packed(&maps.m8[i], sg.packed, sg.ld_packed, sg.N, L.K, 8))
      return kTmaNotApplicable;
    a.seg[i] = TSeg{sg.absmax, sg.ld_absmax, sg.absmax2, sg.gblk_base, sg.gblk_row_stride, sg.offset,
                    sg.y, sg.ldy, rows_total};
    if (L.mode != kTmaSiluMul) {
      rows_total += sg.N;
      a.seg_end_ru[i] = rows_total / 8;
    }
  }
  if (L.mode == kTmaSiluMul) {
    a.ru_total = L.seg[0].N / 8;
    a.seg[1].row_begin = 0;
  } else {
    a.ru_total = rows_total / 8;
  }
  a.N = rows_total;
  if (L.mode == kTmaAllReduce) a.are = L.ar;
  if (static_cast<int64_t>(a.ru_total) * 256 >= (int64_t(1) << 31)) return kTmaNotApplicable;
  if (L.dtype == B2D_F16)
    return L.y_dtype == B2D_F32 ? dispatch_mode<__half, float>(L, maps, a, dev, stream)
                                : dispatch_mode<__half, __half>(L, maps, a, dev, stream);
  return L.y_dtype == B2D_F32 ? dispatch_mode<__nv_bfloat16, float>(L, maps, a, dev, stream)
                              : dispatch_mode<__nv_bfloat16, __nv_bfloat16>(L, maps, a, dev, stream);
}

}  // namespace b2d
