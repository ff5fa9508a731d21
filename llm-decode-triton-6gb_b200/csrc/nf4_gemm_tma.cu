// Fused NF4 dequant + skinny matmul for decode batches (M <= 8) on sm_100a, weights staged by TMA.
// y[M, N] = x[M, K] @ W[N, K]^T with W in bitsandbytes NF4 (replaces the reference's Triton kernel,
// profiling/kernels/nf4_gemm.py:37-64, and its launcher NF4Weight.matmul, nf4_gemm.py:94-106; same
// storage semantics: row-major packed nibbles, even element in the high nibble, one scale per 64
// weights, optional double-quantised scale code2[q] * absmax2[blk / 256] + offset, fp32 accumulation).
//
// At M <= 8 the kernel is bound by instruction issue and the shared-memory pipe, not by HBM: with the
// weights resident in L2 it runs no faster than streaming them. The design therefore spends as few
// instructions per weight byte as the table dequant allows:
//  * Weights: each warp owns a ring of kRing stages of 4 KB (32 rows x 4 blocks of 64 weights) filled
//    by 2-D tensor copies (cp.async.bulk.tensor, 128-byte swizzle) completed on one mbarrier per stage.
//    Lane 0 issues; no per-lane copy instructions; up to 12 KB per warp in flight.
//  * Fragments: lane (g, t) reads rows g and g+8 of a 16-row tile with one 8-byte shared load each:
//    packed bytes [8t, 8t+8) of a block (conflict-free under the swizzle).
//  * Dequant: one byte permute + one 4-byte shared load per packed byte. A 256-entry table maps a
//    packed byte to the pair (code[hi], code[lo]) in the activation dtype, i.e. one tensor-core
//    A-fragment register; entry e, lane l at byte 256 e + 4 l, so every lookup hits 32 distinct banks.
//    The table sits at a 64 KB-aligned shared address, so the one permute that extracts the byte also
//    forms the complete address (lane offset in byte 0, packed byte in byte 1, the table's base in
//    bytes 2-3): no address arithmetic per lookup. The other 128 bytes of each entry hold 32 lane copies
//    of the double-quant table code2. The rest of shared memory is laid out around the table.
//  * MMA: the block scale is factored out of the dot product: four m16n8k16 MMAs per 16-row tile and
//    block accumulate sum_k x_k * code[n_k] from zero, one fp32 FMA per output applies the scale. The
//    reduction axis is permuted so that a lane's 8 packed bytes and its 16 activations of a block cover
//    the same k values: lane (g, t) owns k in [16t, 16t + 16) of each block.
//  * Activations: each warp owns a fixed slice of one or two 4-block K groups for the whole launch; its
//    activations (8 tokens x up to 512 k) sit in registers, loaded once after the dependency wait.
//  * Partition: clusters of 1, 2 or 4 CTAs. A cluster owns a contiguous range of 8-row units (balanced
//    to one unit); its CTAs split the K groups evenly and the warps of a CTA split the CTA's K groups.
//    Rows go in groups of 32 (16 output rows of gate and up in SwiGLU mode) that never straddle a
//    segment. After a group, the warps' partial tiles meet in shared memory (one named barrier, two
//    buffers) and are summed in warp order; the CTAs of a cluster sum theirs through distributed shared
//    memory at the end, in rank order. Results are deterministic.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "nf4_tma.cuh"

namespace b2d {
namespace {

constexpr int kNW = 8;                   // warps per CTA
constexpr int kRing = 3;                 // stages per warp
constexpr int kStage = 4096;             // one stage: 32 rows x 128 bytes (4 blocks)
constexpr int kTmaLutBytes = 64 * 1024;  // 256 entries x 256 B: dequant pairs (bytes 0..127) + code2 (128..255)
constexpr int kMaxGrp = 8;               // row groups per CTA kept for the cluster sum (cs > 1)
constexpr int kEpiStore = 0, kEpiPair = 1, kEpiAllReduce = 2;

struct TmaMaps {
  CUtensorMap m[kTmaMaxSeg];    // boxes of one full group: 32 rows (SwiGLU: 16 rows of each segment) x 128 B
  CUtensorMap m8[kTmaMaxSeg];   // boxes of 8 rows x 128 B (groups of fewer rows)
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
  int M, K;
  int ngk;            // K groups of 4 blocks (K / 256)
  int nseg;
  int static_w;
  int ru_total;       // 8-row units (independent / all-reduce) or units of 8 output rows (SwiGLU)
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

constexpr size_t kSlotFloats = 256;   // one warp's partial tile set: 32 rows x 8 tokens
constexpr uint32_t kRingBytes = kRing * kStage;                      // one warp's ring

// Shared-memory layout around the 64 KB-aligned table: the decoded-scale buffers, exchange buffer and
// mbarriers, then as many warp rings as fit (1 KB aligned) below the table; the remaining rings, the
// partial-tile buffers and the kept sums above it. All addresses are shared-window addresses.
struct Layout {
  uint32_t lut, sbufs, sums, bars, lo0, n_below, slots, cpart, end;
};
__host__ __device__ constexpr uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) & ~(a - 1); }
__host__ __device__ inline Layout make_layout(uint32_t base) {
  Layout L{};
  L.lut = align_up(base + 1, 65536u);   // strictly above the start: the small buffers go first
  L.sbufs = base;
  L.sums = L.sbufs + kNW * 2 * 128 * 4;
  L.bars = L.sums + 2 * kSlotFloats * 4;
  L.lo0 = align_up(L.bars + kNW * kRing * 8, 1024u);
  const uint32_t fit = L.lut > L.lo0 ? (L.lut - L.lo0) / kRingBytes : 0u;
  L.n_below = fit < static_cast<uint32_t>(kNW) ? fit : static_cast<uint32_t>(kNW);
  L.slots = L.lut + kTmaLutBytes + (kNW - L.n_below) * kRingBytes;
  L.cpart = L.slots + 2 * kNW * kSlotFloats * 4;
  L.end = L.cpart + kMaxGrp * kSlotFloats * 4;
  return L;
}
__host__ __device__ inline uint32_t ring_addr(const Layout& L, uint32_t w) {
  return w < L.n_below ? L.lo0 + w * kRingBytes : L.lut + kTmaLutBytes + (w - L.n_below) * kRingBytes;
}
// Dynamic shared memory a launch requests: the layout for the largest dynamic-memory start address
// (the start is 1 KB aligned; the reserved region before it is far below 64 KB), rounded to 1 KB.
constexpr uint32_t kMaxBase = 8192;
uint32_t tma_smem_bytes() {
  uint32_t worst = 0;
  for (uint32_t b = 0; b <= kMaxBase; b += 1024) {
    const Layout L = make_layout(b);
    worst = L.end - b > worst ? L.end - b : worst;
  }
  return worst;
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
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t local_addr, int rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(local_addr), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];\n" : "=f"(v) : "r"(remote) : "memory");
  return v;
}
// Activations are the previous kernel's output: read with coherent loads in volatile asm so that they
// cannot be scheduled above the dependency wait.
__device__ __forceinline__ uint4 ld_act_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p)
               : "memory");
  return v;
}

// A row group: 8-row units [r, r + c) of segment s (SwiGLU mode: units of 8 output rows, s = 0).
struct Grp {
  int r, c, s;
};
template <int EPI>
__device__ __forceinline__ Grp group_at(const TArgs& a, int r, int ru1) {
  constexpr int UPG = EPI == kEpiPair ? 2 : 4;
  Grp gr;
  gr.r = r;
  int s = 0;
#pragma unroll
  for (int i = 0; i < kTmaMaxSeg - 1; ++i) s += (i + 1 < a.nseg && r >= a.seg_end_ru[i]) ? 1 : 0;
  gr.s = EPI == kEpiPair ? 0 : s;
  int e = ru1;
  if (EPI != kEpiPair) e = min(e, a.seg_end_ru[gr.s]);
  gr.c = min(UPG, e - r);
  return gr;
}

// Raw scales of one stage for lane `lane`'s row (row `lane` of the stage): double quant = the four
// code2 indices of the stage's blocks and the row's absmax2 value; plain = four fp32 scales.
template <bool NESTED> struct RawScale;
template <> struct RawScale<true> {
  uint32_t q;
  float a2;
};
template <> struct RawScale<false> {
  float4 f;
};

// Segment and segment-local row of stage row `row` (0..31) of group gr; false past the group's rows.
template <int EPI>
__device__ __forceinline__ bool stage_row(const TArgs& a, const Grp& gr, int row, int& s, int64_t& seg_row) {
  if (EPI == kEpiPair) {
    s = row >> 4;   // rows 0..15 gate, 16..31 up
    const int rr = row & 15;
    seg_row = 8ll * gr.r + rr;
    return rr < 8 * gr.c;
  }
  s = gr.s;
  seg_row = 8ll * gr.r + row - a.seg[gr.s].row_begin;
  return row < 8 * gr.c;
}

template <bool NESTED, int EPI>
__device__ __forceinline__ void load_raw(RawScale<NESTED>& rs, const TArgs& a, const Grp& gr, int kg, int lane) {
  int s;
  int64_t row;
  const bool ok = stage_row<EPI>(a, gr, lane, s, row);
  const TSeg& sg = a.seg[s];
  if constexpr (NESTED) {
    rs.q = 0;
    rs.a2 = 0.f;
    if (!ok) return;
    // 4 code2 indices: 4-byte aligned (the host checks the table, its row stride and the block offsets)
    rs.q = __ldg(reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(sg.absmax) + row * sg.ld_absmax +
                                                   4 * kg));
    rs.a2 = __ldg(sg.absmax2 + ((sg.gblk_base + row * sg.gblk_row_stride + 4 * kg) >> 8));
  } else {
    rs.f = make_float4(0.f, 0.f, 0.f, 0.f);
    if (!ok) return;
    rs.f = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(sg.absmax) + row * sg.ld_absmax + 4 * kg));
  }
}

// Decoded fp32 block scales of lane's row into the warp's scale buffer (16 bytes per row). Rows past
// the group decode to finite values (their outputs are never stored).
template <bool NESTED>
__device__ __forceinline__ void decode_scales(const RawScale<NESTED>& rs, float* sb, uint32_t lane_c2, float off,
                                              int lane) {
  float4 v;
  if constexpr (NESTED) {
    auto c2 = [&](uint32_t sel) {
      float f;
      asm volatile("ld.shared.f32 %0, [%1];\n" : "=f"(f) : "r"(__byte_perm(rs.q, lane_c2, sel)) : "memory");
      return f;
    };
    v.x = __fadd_rn(__fmul_rn(c2(0x7604u), rs.a2), off);
    v.y = __fadd_rn(__fmul_rn(c2(0x7614u), rs.a2), off);
    v.z = __fadd_rn(__fmul_rn(c2(0x7624u), rs.a2), off);
    v.w = __fadd_rn(__fmul_rn(c2(0x7634u), rs.a2), off);
  } else {
    v = rs.f;
  }
  *reinterpret_cast<float4*>(sb + lane * 4) = v;
}

// Table lookup of byte K of `word`: lane_lut = table base | 4 lane; sel = 0x76K4 keeps the base's bytes
// 2-3 and the lane offset and puts the packed byte in byte 1. The address depends on stage data read
// after the stage's barrier wait, so the load cannot move above the table build.
__device__ __forceinline__ uint32_t lut_at(uint32_t word, uint32_t lane_lut, uint32_t sel) {
  uint32_t v;
  asm("ld.shared.b32 %0, [%1];\n" : "=r"(v) : "r"(__byte_perm(word, lane_lut, sel)));
  return v;
}

// One stage (2 row tiles x 4 blocks) into acc[2][4]. No guards: rows the copy did not fill hold stale
// packed bytes (every byte is a valid table index, so the products are finite) whose scales are zero.
// Fragment row g of a 16-row tile is stage row rho(g) = 2 (g & 3) + (g >> 2) of the tile (and row
// g + 8 is rho(g) + 8): the 16 lanes of each half-warp then read rows of one parity, whose swizzled
// 16-byte chunks of a block are all distinct, so the 8-byte fragment loads are conflict-free.
__device__ __forceinline__ int rho(int g) { return ((g & 3) << 1) | (g >> 2); }

// One stage (2 row tiles x 4 blocks) into acc[2][4]. No guards: rows the copy did not fill hold stale
// packed bytes (every byte is a valid table index, so the products are finite) whose outputs are never
// stored.
template <typename T>
__device__ __forceinline__ void compute_stage(uint32_t stage_s, const uint4 (&xr)[4][2], const float* sb, int rg,
                                              int tq, float (&acc)[2][4], uint32_t lane_lut) {
#pragma unroll
  for (int tt = 0; tt < 2; ++tt) {
    const float4 s0 = *reinterpret_cast<const float4*>(sb + (16 * tt + rg) * 4);
    const float4 s1 = *reinterpret_cast<const float4*>(sb + (16 * tt + 8 + rg) * 4);
    const float sl[4] = {s0.x, s0.y, s0.z, s0.w}, sh[4] = {s1.x, s1.y, s1.z, s1.w};
    const uint32_t r0 = stage_s + (16 * tt + rg) * 128 + 8 * (tq & 1);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const uint32_t co = static_cast<uint32_t>(((2 * jj + (tq >> 1)) ^ rg) << 4);
      const uint2 wl = lds64(r0 + co);          // row rg: packed bytes [8 tq, 8 tq + 8) of block jj
      const uint2 wh = lds64(r0 + 1024 + co);   // row rg + 8
      float c[4];
      Mma<T>::run0(c, lut_at(wl.x, lane_lut, 0x7604u), lut_at(wh.x, lane_lut, 0x7604u),
                   lut_at(wl.x, lane_lut, 0x7614u), lut_at(wh.x, lane_lut, 0x7614u), xr[jj][0].x, xr[jj][0].y);
      Mma<T>::run(c, lut_at(wl.x, lane_lut, 0x7624u), lut_at(wh.x, lane_lut, 0x7624u),
                  lut_at(wl.x, lane_lut, 0x7634u), lut_at(wh.x, lane_lut, 0x7634u), xr[jj][0].z, xr[jj][0].w);
      Mma<T>::run(c, lut_at(wl.y, lane_lut, 0x7604u), lut_at(wh.y, lane_lut, 0x7604u),
                  lut_at(wl.y, lane_lut, 0x7614u), lut_at(wh.y, lane_lut, 0x7614u), xr[jj][1].x, xr[jj][1].y);
      Mma<T>::run(c, lut_at(wl.y, lane_lut, 0x7624u), lut_at(wh.y, lane_lut, 0x7624u),
                  lut_at(wl.y, lane_lut, 0x7634u), lut_at(wh.y, lane_lut, 0x7634u), xr[jj][1].z, xr[jj][1].w);
      acc[tt][0] = fmaf(sl[jj], c[0], acc[tt][0]);
      acc[tt][1] = fmaf(sl[jj], c[1], acc[tt][1]);
      acc[tt][2] = fmaf(sh[jj], c[2], acc[tt][2]);
      acc[tt][3] = fmaf(sh[jj], c[3], acc[tt][3]);
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

// Final output of thread (warp, lane) for group gr: v = its element of the summed tile set ([fragment
// row][token]: token t = lane & 7, fragment row fr = 4 warp + lane / 8, i.e. stage row
// 8 (fr / 8) + rho(fr & 7)); SwiGLU: output row r < 16 from gate row r (v) and up row 16 + r (up);
// all-reduce: token pairs packed into flag-in-word pushes.
template <typename OT, int EPI>
__device__ __forceinline__ void store_group(const TArgs& a, const Grp& gr, float v, float up, int warp, int lane,
                                            uint32_t epoch) {
  const int t = lane & 7, fr = 4 * warp + (lane >> 3), r = (fr & ~7) | rho(fr & 7);
  if constexpr (EPI == kEpiPair) {
    if (r < 16 && t < a.M && r < 8 * gr.c)
      static_cast<OT*>(a.seg[0].y)[t * a.seg[0].ldy + 8ll * gr.r + r] = swiglu<OT>(v, up);
  } else if constexpr (EPI == kEpiAllReduce) {
    const float next = __shfl_down_sync(0xffffffffu, v, 1);
    if constexpr (!std::is_same<OT, float>::value) {
      if ((t & 1) == 0 && t < a.M && r < 8 * gr.c) {
        const int64_t grow = 8ll * gr.r + r;   // one segment: launch rows are output rows
        const uint64_t word = (static_cast<uint64_t>(epoch) << 32) | Dt<OT>::pack2(v, next);
        const int64_t w = static_cast<int64_t>(t >> 1) * a.N + grow;
        for (int p = 0; p < a.are.world; ++p) st_word(ar_slot(a.are, p, a.are.rank, epoch) + w, word);
      }
    }
  } else {
    if (t < a.M && r < 8 * gr.c) {
      const TSeg& sg = a.seg[gr.s];
      static_cast<OT*>(sg.y)[t * sg.ldy + 8ll * gr.r - sg.row_begin + r] = Dt<OT>::from_f32(v);
    }
  }
}

// SwiGLU needs the up-row sum held by another warp: exchange through a double-buffered array (by group
// parity, so one barrier per group suffices), then store.
template <typename OT, int EPI>
__device__ __forceinline__ void finish_group(const TArgs& a, const Grp& gr, float v, float* sums, int parity,
                                             int warp, int lane, uint32_t epoch) {
  float up = 0.f;
  if constexpr (EPI == kEpiPair) {
    float* sm = sums + parity * kSlotFloats;
    sm[32 * warp + lane] = v;
    named_bar(2, kNW * 32);
    if (warp < 4) up = sm[32 * warp + lane + 128];
  }
  store_group<OT, EPI>(a, gr, v, up, warp, lane, epoch);
}

template <typename T, typename OT, bool NESTED, int EPI>
__global__ void __launch_bounds__(kNW * 32, 1) nf4_tma_kernel(const __grid_constant__ TmaMaps maps,
                                                              const __grid_constant__ TArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t base = smem_u32(smem);
  uint32_t dyn_bytes;
  asm("mov.u32 %0, %%dynamic_smem_size;\n" : "=r"(dyn_bytes));
  const Layout lay = make_layout(base);
  // The fragment reads assume the 128-byte swizzle pattern relative to 1024-byte aligned stages, and the
  // layout must fit the launch's shared memory: otherwise the launch records an error and does nothing
  // (the same for every CTA, so no cluster barrier is left waiting).
  if ((base & 1023u) != 0 || lay.end > base + dyn_bytes) {
    if (tid == 0 && a.err) atomicAdd(a.err, 1 << 16);
    return;
  }
  auto at = [&](uint32_t addr) { return smem + (addr - base); };
  float* slots = reinterpret_cast<float*>(at(lay.slots));   // [2][kNW][32 rows][8 tokens]
  float* sbufs = reinterpret_cast<float*>(at(lay.sbufs));   // [kNW][2][32 rows][4]
  float* cpart = reinterpret_cast<float*>(at(lay.cpart));   // [kMaxGrp][32 rows][8 tokens]
  float* sums = reinterpret_cast<float*>(at(lay.sums));     // [2][32 rows][8 tokens]
  uint8_t* lut = at(lay.lut);
  const int g = lane >> 2, tq = lane & 3, rg = rho(g);
  const uint32_t lane4 = static_cast<uint32_t>(lane) * 4u;
  const uint32_t lane_lut = lay.lut | lane4;
  const uint32_t lane_c2 = lay.lut | (128u + lane4);

  // ---- partition (32-bit math; the host keeps ru_total * clusters and ngk * cs below 2^31)
  const int cs = cluster_size(), q = cluster_rank(), cl = cluster_index(), ncl = cluster_count();
  const int ru0 = cl * a.ru_total / ncl, ru1 = (cl + 1) * a.ru_total / ncl;
  const int kg0 = q * a.ngk / cs, kg1 = (q + 1) * a.ngk / cs;
  const int wk0 = kg0 + warp * (kg1 - kg0) / kNW, wk1 = kg0 + (warp + 1) * (kg1 - kg0) / kNW;
  const int nst = wk1 - wk0;   // stages per row group for this warp: 0, 1 or 2 (host)

  const uint32_t ring_s = ring_addr(lay, warp);
  const uint32_t bar_s = lay.bars + warp * kRing * 8;
  float* sbw = sbufs + warp * 2 * 128;
  if (lane == 0) {
    for (int s = 0; s < kRing; ++s) mbar_init(bar_s + 8 * s, 1);
    fence_mbar_init();
  }
  __syncwarp();

  // ---- issue side (lane 0): stage u = (group, sub-stage) in consumption order
  Grp gi = group_at<EPI>(a, ru0, ru1);   // group of the next stage to issue
  int si = 0;
  int iu = 0;
  auto issue_next = [&]() {
    if (nst == 0 || gi.r >= ru1) return;
    const uint32_t st = ring_s + (iu % kRing) * kStage, bar = bar_s + 8 * (iu % kRing);
    const int xk = (wk0 + si) * 128;
    if (EPI == kEpiPair) {
      mbar_expect_tx(bar, static_cast<uint32_t>(gi.c) * 2048u);
      if (gi.c == 2) {
        tma_load_2d(st, &maps.m[0], xk, 8 * gi.r, bar);
        tma_load_2d(st + 2048, &maps.m[1], xk, 8 * gi.r, bar);
      } else {
        tma_load_2d(st, &maps.m8[0], xk, 8 * gi.r, bar);
        tma_load_2d(st + 2048, &maps.m8[1], xk, 8 * gi.r, bar);
      }
    } else {
      mbar_expect_tx(bar, static_cast<uint32_t>(gi.c) * 1024u);
      const int y = 8 * gi.r - a.seg[gi.s].row_begin;
      if (gi.c == 4) {
        tma_load_2d(st, &maps.m[gi.s], xk, y, bar);
      } else {
        for (int i = 0; i < gi.c; ++i) tma_load_2d(st + 1024 * i, &maps.m8[gi.s], xk, y + 8 * i, bar);
      }
    }
    ++iu;
    if (++si == nst) {
      si = 0;
      gi = group_at<EPI>(a, gi.r + gi.c, ru1);
    }
  };

  // Weights start streaming before the table is built: at once when they do not depend on the
  // preceding kernel (static weights), else right after the dependency wait. The first group's raw
  // scales are requested at the same time.
  if (!a.static_w) pdl_wait();
  if (lane == 0)
    for (int k = 0; k < kRing; ++k) issue_next();
  Grp gc = group_at<EPI>(a, ru0, ru1);   // group being computed
  RawScale<NESTED> raw[2];
  if (nst > 0) load_raw<NESTED, EPI>(raw[0], a, gc, wk0, lane);
  if (nst > 1) load_raw<NESTED, EPI>(raw[1], a, gc, wk0 + 1, lane);

  // ---- dequant table + code2 lane copies: thread e builds entry e (8 x 16-byte stores per half, 4
  // distinct 16-byte bank groups per 8 lanes: 4 wavefronts per instruction)
  {
    const float my_code = a.code_by_value ? a.code_v[lane & 15] : __ldg(a.code_dev + (lane & 15));
    const int e = tid;   // kNW * 32 == 256 entries
    const float hi = __shfl_sync(0xffffffffu, my_code, (e >> 4) & 15);
    const float lo = __shfl_sync(0xffffffffu, my_code, e & 15);
    const uint32_t val = Dt<T>::pack2(hi, lo);
    uint4* entry = reinterpret_cast<uint4*>(lut + e * 256);
    const uint4 v4 = make_uint4(val, val, val, val);
#pragma unroll
    for (int i = 0; i < 8; ++i) entry[(i + lane) & 7] = v4;
    if (NESTED) {
      const uint32_t c2 = __float_as_uint(__ldg(a.code2 + e));
      const uint4 c4 = make_uint4(c2, c2, c2, c2);
#pragma unroll
      for (int i = 0; i < 8; ++i) entry[8 + ((i + lane) & 7)] = c4;
    }
  }
  __syncthreads();
  pdl_wait();   // activations and outputs are stream-ordered from here
  const uint32_t epoch = EPI == kEpiAllReduce ? ar_epoch(a.are) : 0u;

  // ---- this warp's activations: 8 tokens x its K groups, lane (g, tq) -> token g, k 16 tq .. 16 tq + 15
  // of every block
  uint4 xr[2][4][2];
  {
    const int tok = g < a.M ? g : 0;   // rows past M read token 0; their outputs are never stored
    const T* xp = static_cast<const T*>(a.x) + static_cast<int64_t>(tok) * a.ldx + wk0 * 256 + 16 * tq;
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (s < nst) {
          xr[s][j][0] = ld_act_u4(xp + s * 256 + j * 64);
          xr[s][j][1] = ld_act_u4(xp + s * 256 + j * 64 + 8);
        } else {
          xr[s][j][0] = xr[s][j][1] = make_uint4(0, 0, 0, 0);
        }
      }
  }

  int u = 0;      // stages consumed (ring slot u % kRing, phase (u / kRing) & 1)
  int nb = 0;     // row groups done
  // double-quant offset of the lane's scale row (SwiGLU: gate rows 0..15, up rows 16..31)
  float off = NESTED ? a.seg[EPI == kEpiPair ? (lane >> 4) : gc.s].offset : 0.f;
  while (gc.r < ru1) {
    const Grp gn = group_at<EPI>(a, gc.r + gc.c, ru1);
    float acc[2][4] = {};
#define B2D_TMA_STAGE(S)                                                                                      \
    if (S < nst) {                                                                                            \
      float* sb = sbw + (u & 1) * 128;                                                                        \
      decode_scales<NESTED>(raw[S], sb, lane_c2, off, lane);                                             \
      if (gn.r < ru1) load_raw<NESTED, EPI>(raw[S], a, gn, wk0 + S, lane);   /* next group's, one ahead */    \
      __syncwarp();                                                                                           \
      const uint32_t slot = u % kRing;                                                                        \
      mbar_wait(bar_s + 8 * slot, static_cast<uint32_t>((u / kRing) & 1), a.err);                             \
      compute_stage<T>(ring_s + slot * kStage, xr[S], sb, rg, tq, acc, lane_lut);                           \
      __syncwarp();                                                                                           \
      if (lane == 0) issue_next();   /* the stage's bytes were consumed by the MMAs above */               \
      ++u;                                                                                                    \
    }
    B2D_TMA_STAGE(0) B2D_TMA_STAGE(1)
#undef B2D_TMA_STAGE
    // this warp's partial tiles, [fragment row][token] (fragment row 16 tt + 8 h + g, token 2 tq + i)
    float* sl = slots + ((nb & 1) * kNW + warp) * kSlotFloats;
#pragma unroll
    for (int tt = 0; tt < 2; ++tt) {
      *reinterpret_cast<float2*>(sl + (16 * tt + g) * 8 + 2 * tq) = make_float2(acc[tt][0], acc[tt][1]);
      *reinterpret_cast<float2*>(sl + (16 * tt + 8 + g) * 8 + 2 * tq) = make_float2(acc[tt][2], acc[tt][3]);
    }
    named_bar(1, kNW * 32);
    // the CTA's sum over its warps (warp order): thread -> element 32 warp + lane of the tile set
    const float* sp = slots + (nb & 1) * kNW * kSlotFloats + 32 * warp + lane;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kNW; ++w) v += sp[w * kSlotFloats];
    if (cs == 1) finish_group<OT, EPI>(a, gc, v, sums, nb & 1, warp, lane, epoch);
    else cpart[nb * kSlotFloats + 32 * warp + lane] = v;
    ++nb;
    if (NESTED && EPI != kEpiPair && gn.s != gc.s) off = a.seg[gn.s].offset;
    gc = gn;
  }
  if (cs == 1) return;
  // ---- the cluster's sum over its CTAs (rank order); group b is stored by CTA b % cs
  cluster_sync();
  {
    Grp gb = group_at<EPI>(a, ru0, ru1);
    for (int b = 0; gb.r < ru1; ++b, gb = group_at<EPI>(a, gb.r + gb.c, ru1)) {
      if (b % cs != q) continue;
      const uint32_t la = smem_u32(cpart + b * kSlotFloats + 32 * warp + lane);
      float v = 0.f;
      for (int r = 0; r < cs; ++r) v += ld_dsmem_f32(la, r);
      finish_group<OT, EPI>(a, gb, v, sums, b & 1, warp, lane, epoch);
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
  int cs, ncl;
};

template <typename T, typename OT, bool NESTED, int EPI>
struct TmaKernel {
  static size_t smem() {
    static const size_t bytes = tma_smem_bytes();
    return bytes;
  }
  // Max active clusters of size 1, 2, 4 for this instantiation on the current device (queried once).
  static const int* max_clusters(int dev) {
    static int table[64][3];
    static std::once_flag once[64];
    std::call_once(once[dev], [&] {
      auto kern = nf4_tma_kernel<T, OT, NESTED, EPI>;
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem())) !=
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
        cfg.blockDim = dim3(kNW * 32);
        cfg.dynamicSmemBytes = smem();
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
    cfg.blockDim = dim3(kNW * 32);
    cfg.dynamicSmemBytes = smem();
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
    const cudaError_t e = cudaLaunchKernelEx(&cfg, nf4_tma_kernel<T, OT, NESTED, EPI>, maps, a);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return B2D_ERR_LAUNCH;
    }
    return launch_status();
  }
};

// Row groups a CTA of a cluster owning `units` 8-row units walks: at most ceil(units / upg) plus one
// per segment boundary inside the range.
int groups_bound(int units, int upg, int nseg) { return (units + upg - 1) / upg + nseg - 1; }

// Picks the cluster size: every warp's share of its CTA's K groups must be at most 2 (the activations
// stay in registers), a cluster's row groups must fit the kept sums when cs > 1, and among those the
// configuration with the least work on the busiest CTA (row units per cluster x K groups per CTA) wins;
// ties go to the smaller cluster.
template <class K>
bool choose(const TArgs& a, int dev, TmaConfig* out, int upg) {
  const int* mc = K::max_clusters(dev);
  int64_t best = -1;
  for (int i = 0; i < 3; ++i) {
    const int cs = 1 << i;
    if (mc[i] <= 0) continue;
    const int kc = (a.ngk + cs - 1) / cs;
    if ((kc + kNW - 1) / kNW > 2) continue;
    const int ncl = mc[i] < a.ru_total ? mc[i] : a.ru_total;
    const int per = (a.ru_total + ncl - 1) / ncl;
    if (cs > 1 && groups_bound(per, upg, a.nseg) > kMaxGrp) continue;
    const int64_t work = static_cast<int64_t>(per) * kc;
    if (best < 0 || work < best) {
      best = work;
      *out = TmaConfig{cs, ncl};
    }
  }
  return best >= 0;
}

template <typename T, typename OT, bool NESTED, int EPI>
int dispatch(const TmaMaps& maps, const TArgs& a, int dev, bool pdl, cudaStream_t s) {
  using K = TmaKernel<T, OT, NESTED, EPI>;
  TmaConfig c;
  if (!choose<K>(a, dev, &c, EPI == kEpiPair ? 2 : 4)) return kTmaNotApplicable;
  return K::launch(maps, a, c, pdl, s);
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
  if (L.M < 1 || L.M > 8 || L.K < 256 || L.K % 256 || L.nseg < 1 || L.nseg > kTmaMaxSeg) return kTmaNotApplicable;
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
  a.ngk = L.K / 256;
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
    // every stage's four scales of a row: one aligned 4-byte (nested) or 16-byte (plain) load, inside one
    // 256-block group of absmax2
    if (L.nested) {
      if (!aligned(sg.absmax, 4) || sg.ld_absmax % 4 || sg.code2 != L.seg[0].code2 || !sg.code2 || !sg.absmax2 ||
          sg.gblk_base % 4 || sg.gblk_row_stride % 4)
        return kTmaNotApplicable;
    } else if (!aligned(sg.absmax, 16) || sg.ld_absmax % 4) {
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
    a.seg_end_ru[0] = a.seg_end_ru[1] = a.ru_total;
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
