// Fused NF4 dequant + skinny matmul for sm_100a: y[M,N] = x[M,K] @ W[N,K]^T, W in bitsandbytes NF4.
//
// Replaces the reference's Triton kernel (profiling/kernels/nf4_gemm.py:37-64) and its launcher
// NF4Weight.matmul (nf4_gemm.py:94-106). Same storage semantics: row-major packed nibbles, even
// element in the high nibble, one scale per 64 weights, optional double-quant scale
// code2[q]*absmax2[blk/256]+offset (nf4_gemm.py:48-56); fp32 accumulation.
//
// Design (HBM-bound: ~0.52 B of weight state per weight, 2*M flops per weight):
//  * Persistent grid, one CTA per SM. The work is the list of (row group, chunk of CB 64-weight
//    blocks) units in row-group-major order; every CTA gets an equal contiguous slice and every warp
//    an equal contiguous sub-slice, so all SMs stream the same number of bytes for any (N, K). A row
//    group split between warps is summed in shared memory, one split between CTAs through a small
//    global workspace; the CTA that finishes a shared group last (acquire-release atomic counter)
//    adds the partials in CTA order, so results are deterministic.
//  * Weights go global -> registers with 8-byte streaming loads (no shared-memory staging: the
//    shared-memory pipe is reserved for the dequant table), double-buffered one unit ahead; the
//    first unit's loads are issued before the table is built.
//  * Dequant: a 256-entry table maps one packed byte to the pair (code[hi], code[lo]) in the
//    activation dtype, i.e. directly to one tensor-core A-fragment register. Entry e, lane l lives
//    at byte 256*e + 4*l, so lookups never bank-conflict and one byte permute of the packed word
//    with 4*lane produces the address.
//  * The per-block scale is factored out of the dot product: the four m16n8k16 MMAs of one block
//    accumulate sum_k x_k*code[n_k] from zero, and the fp32 block scale multiplies that partial
//    into the running fp32 accumulator (one FMA per output element per block).
//  * The MMA reduction dimension is permuted so that each thread's 8 bytes of a block row are
//    contiguous in memory and the matching 16 activations are contiguous too:
//    thread (g, t) at k-step s owns bytes 8t+2s, 8t+2s+1 of its block row = k offsets 16t+4s+{0..3}.
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "nf4_tc5.cuh"
#include "nf4_tma.cuh"

namespace b2d {

namespace {

constexpr int kLutEntryBytes = 256;                 // 32 lanes x 4 B used; stride chosen for the permute
constexpr int kLutBytes = 256 * kLutEntryBytes;     // 64 KB
constexpr int kCode2Bytes = 256 * 4;

struct Nf4View {
  const uint8_t* packed;
  int64_t ld_packed;
  const void* absmax;
  int64_t ld_absmax;
  const float* code2;
  const float* absmax2;
  float offset;
  int64_t gblk_base;
  int64_t gblk_row_stride;
  const float* code;
};

constexpr int kMaxSeg = 4;
struct SegView {
  Nf4View w;
  void* y;
  int64_t ldy;
};

struct GemmArgs {
  const void* x;
  int64_t ldx;
  Nf4View w;
  void* y;
  int64_t ldy;
  int M, N, K;
  int upg;           // units (chunks of CB blocks) per row group = K / (64 * CB)
  int groups;        // N / (16 * RT)
  int total;         // groups * upg
  float* partials;   // [grid][2][E]
  int* counters;     // [groups]
  // Segmented launches (pipelined kernel only): the row groups of several weights sharing x, in
  // order. Single-weight launches use one segment equal to (w, y, ldy).
  int nseg;                  // 1..kMaxSeg
  int pair;                  // 1: segments 0/1 interleaved per group, epilogue silu(seg0) * seg1
  int static_w;              // 1: weights may be read before the preceding kernel completes
  int code_by_value;         // 1: code_v holds segment 0's 16 codebook values (no device read)
  float code_v[16];
  int ar;                    // 1: the output goes to every peer as all-reduce words (tensor parallel)
  ArPeers are;
  int seg_end[kMaxSeg];      // exclusive end (in row groups) of each segment
  SegView seg[kMaxSeg];
};

// One unit of work for one thread, loaded a unit ahead: its weight bytes, the raw per-block scales
// of its rows and (for M <= 8) the activations of the unit's first block.
template <int RT, int NT, int CB, bool NESTED>
struct WBuf {
  uint2 w[RT][2][CB];                       // rows g, g+8 of each 16-row tile; 8 bytes per block
  uint32_t sq[RT][2][NESTED ? 1 : CB];      // double quant: CB uint8 indices packed; else fp32 bits
  float a2[RT][2];                          // double quant: absmax2 of the row's 256-block group
  uint4 x0[NT == 1 ? 1 : 1][2];             // activations of block 0 (used when NT == 1)
};

template <typename T, int NT>
__device__ __forceinline__ void load_x(uint4 (&xv)[NT][2], const GemmArgs& a, int blk, int g, int tq) {
  const T* x = static_cast<const T*>(a.x);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int tok = nt * 8 + g;
    if (tok < a.M) {
      const T* p = x + tok * a.ldx + blk * 64 + tq * 16;
      xv[nt][0] = ldg_u4(p);
      xv[nt][1] = ldg_u4(p + 8);
    } else {
      xv[nt][0] = make_uint4(0, 0, 0, 0);
      xv[nt][1] = make_uint4(0, 0, 0, 0);
    }
  }
}

template <typename T, int RT, int NT, int CB, bool NESTED>
__device__ __forceinline__ void load_w(WBuf<RT, NT, CB, NESTED>& b, const GemmArgs& a, int grp, int unit, int g,
                                       int tq) {
#pragma unroll
  for (int rt = 0; rt < RT; ++rt) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t row = static_cast<int64_t>(grp) * (16 * RT) + rt * 16 + h * 8 + g;
      const uint8_t* p = a.w.packed + row * a.w.ld_packed + unit * (CB * 32) + tq * 8;
#pragma unroll
      for (int j = 0; j < CB; ++j) b.w[rt][h][j] = ldg_stream_u2(p + 32 * j);
      const int64_t bi = row * a.w.ld_absmax + static_cast<int64_t>(unit) * CB;
      if (NESTED) {
        const uint8_t* q = static_cast<const uint8_t*>(a.w.absmax) + bi;
        b.sq[rt][h][0] = CB == 4 ? __ldg(reinterpret_cast<const uint32_t*>(q)) : static_cast<uint32_t>(__ldg(q));
        // a chunk never straddles a 256-block group of absmax2 (the host guarantees 4-alignment)
        b.a2[rt][h] = __ldg(a.w.absmax2 + ((a.w.gblk_base + row * a.w.gblk_row_stride + unit * CB) >> 8));
      } else {
        const float* sp = static_cast<const float*>(a.w.absmax) + bi;
        if (CB == 4) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(sp));
          b.sq[rt][h][0] = __float_as_uint(v.x);
          b.sq[rt][h][CB > 1 ? 1 : 0] = __float_as_uint(v.y);
          b.sq[rt][h][CB > 2 ? 2 : 0] = __float_as_uint(v.z);
          b.sq[rt][h][CB > 3 ? 3 : 0] = __float_as_uint(v.w);
        } else {
          b.sq[rt][h][0] = __float_as_uint(__ldg(sp));
        }
      }
    }
  }
  if (NT == 1) {
    uint4 (&x0)[1][2] = reinterpret_cast<uint4 (&)[1][2]>(b.x0);
    load_x<T, 1>(x0, a, unit * CB, g, tq);
  }
}

__device__ __forceinline__ uint32_t lut_lookup(const uint8_t* lut, uint32_t word, uint32_t lane4, uint32_t sel) {
  return *reinterpret_cast<const uint32_t*>(lut + __byte_perm(word, lane4, sel));
}

template <typename T, int RT, int NT, int CB, bool NESTED>
__device__ __forceinline__ void compute_unit(const WBuf<RT, NT, CB, NESTED>& b, const GemmArgs& a, int unit,
                                             float (&acc)[RT][NT][4], const uint8_t* lut, uint32_t lane4,
                                             const float* code2_s, int g, int tq) {
  uint4 xv[NT][2], xn[NT][2];
  if (NT == 1) {
#pragma unroll
    for (int i = 0; i < 2; ++i) xv[0][i] = b.x0[0][i];
  } else {
    load_x<T, NT>(xv, a, unit * CB, g, tq);
  }
#pragma unroll
  for (int j = 0; j < CB; ++j) {
    if (j + 1 < CB) load_x<T, NT>(xn, a, unit * CB + j + 1, g, tq);   // next block's activations
#pragma unroll
    for (int rt = 0; rt < RT; ++rt) {
      float sc[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (NESTED) {
          const uint32_t q = CB == 4 ? (b.sq[rt][h][0] >> (8 * j)) & 0xFF : b.sq[rt][h][0];
          sc[h] = __fadd_rn(__fmul_rn(code2_s[q], b.a2[rt][h]), a.w.offset);
        } else {
          sc[h] = __uint_as_float(b.sq[rt][h][NESTED ? 0 : j]);
        }
      }
      float c[NT][4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const uint32_t wg = (s < 2) ? b.w[rt][0][j].x : b.w[rt][0][j].y;
        const uint32_t wh = (s < 2) ? b.w[rt][1][j].x : b.w[rt][1][j].y;
        const uint32_t sel0 = (s & 1) ? 0x5524u : 0x5504u;   // byte 2(s&1) into bits 8..15, 4*lane below
        const uint32_t sel1 = (s & 1) ? 0x5534u : 0x5514u;   // byte 2(s&1)+1
        const uint32_t a0 = lut_lookup(lut, wg, lane4, sel0);
        const uint32_t a2 = lut_lookup(lut, wg, lane4, sel1);
        const uint32_t a1 = lut_lookup(lut, wh, lane4, sel0);
        const uint32_t a3 = lut_lookup(lut, wh, lane4, sel1);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv[nt][0]);
          if (s == 0) Mma<T>::run0(c[nt], a0, a1, a2, a3, xw[0], xw[1]);
          else Mma<T>::run(c[nt], a0, a1, a2, a3, xw[2 * s], xw[2 * s + 1]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        acc[rt][nt][0] = fmaf(sc[0], c[nt][0], acc[rt][nt][0]);
        acc[rt][nt][1] = fmaf(sc[0], c[nt][1], acc[rt][nt][1]);
        acc[rt][nt][2] = fmaf(sc[1], c[nt][2], acc[rt][nt][2]);
        acc[rt][nt][3] = fmaf(sc[1], c[nt][3], acc[rt][nt][3]);
      }
    }
    if (j + 1 < CB) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) { xv[nt][0] = xn[nt][0]; xv[nt][1] = xn[nt][1]; }
    }
  }
}

// Store a finished 16*RT-row group held in fragment order (thread g,t owns rows g, g+8 of each
// tile and tokens 2t, 2t+1 of each n8 tile).
template <typename OT, int RT, int NT>
__device__ __forceinline__ void store_group(const GemmArgs& a, int grp, const float (&v)[RT][NT][4],
                                            int g, int tq) {
  OT* y = static_cast<OT*>(a.y);
#pragma unroll
  for (int rt = 0; rt < RT; ++rt) {
    const int64_t r0 = static_cast<int64_t>(grp) * (16 * RT) + rt * 16 + g;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int t0 = nt * 8 + 2 * tq;
      if (t0 < a.M) {
        y[t0 * a.ldy + r0] = Dt<OT>::from_f32(v[rt][nt][0]);
        y[t0 * a.ldy + r0 + 8] = Dt<OT>::from_f32(v[rt][nt][2]);
      }
      if (t0 + 1 < a.M) {
        y[(t0 + 1) * a.ldy + r0] = Dt<OT>::from_f32(v[rt][nt][1]);
        y[(t0 + 1) * a.ldy + r0 + 8] = Dt<OT>::from_f32(v[rt][nt][3]);
      }
    }
  }
}

__device__ __forceinline__ int seg_of(const GemmArgs& a, int grp) {
  int s = 0;
#pragma unroll
  for (int i = 0; i < kMaxSeg - 1; ++i) s += (i + 1 < a.nseg && grp >= a.seg_end[i]) ? 1 : 0;
  return s;
}

// SwiGLU in the model dtype, as a Mistral MLP computes it: act_fn(gate_proj(x)) * up_proj(x) with
// every intermediate rounded to OT.
template <typename OT>
__device__ __forceinline__ OT silu_mul(float gate, float up) {
  const float gq = Dt<OT>::to_f32(Dt<OT>::from_f32(gate));
  const float sq = Dt<OT>::to_f32(Dt<OT>::from_f32(gq / (1.0f + expf(-gq))));
  return Dt<OT>::from_f32(sq * Dt<OT>::to_f32(Dt<OT>::from_f32(up)));
}

// store_group for segmented launches (32-row groups): plain segments write their own output; in
// paired mode tile 0 holds rows of segment 0 and tile 1 the same rows of segment 1, and the
// output (segment 0's y) receives silu(tile 0) * tile 1.
// Epilogue kinds of the pipelined kernel, one instantiation each (an epilogue's code and registers
// stay out of the other launches).
constexpr int kEpiStore = 0, kEpiAllReduce = 1;

// All-reduce epilogue (one segment): the partial output rounded to OT, written as flag-in-word words
// (two tokens of one row per word: word (t/2)*N + row) into this rank's slot of every peer's buffer;
// the consumer (b2d_allreduce_add_rmsnorm) sums the world's slots.
template <typename OT, int NT>
__device__ __forceinline__ void store_allreduce(const GemmArgs& a, int grp, const float (&v)[2][NT][4], int g, int tq,
                                                uint32_t e) {
  const int64_t base = static_cast<int64_t>(grp) * 32 + g;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int tp = nt * 4 + tq;   // token pair (2tp, 2tp + 1)
    if (2 * tp >= a.M) continue;
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int64_t w = tp * static_cast<int64_t>(a.N) + base + rt * 16 + h * 8;
        const uint64_t word = (static_cast<uint64_t>(e) << 32) |
                              Dt<OT>::pack2(v[rt][nt][2 * h], v[rt][nt][2 * h + 1]);
        for (int p = 0; p < a.are.world; ++p) st_word(ar_slot(a.are, p, a.are.rank, e) + w, word);
      }
  }
}

template <typename OT, int NT, int EPI = kEpiStore>
__device__ __forceinline__ void store_seg(const GemmArgs& a, int grp, const float (&v)[2][NT][4], int g, int tq,
                                          uint32_t epoch = 0) {
  if constexpr (EPI == kEpiAllReduce) {
    if constexpr (!std::is_same<OT, float>::value) store_allreduce<OT, NT>(a, grp, v, g, tq, epoch);
    return;
  }
  if (a.pair) {
    OT* y = static_cast<OT*>(a.seg[0].y);
    const int64_t ldy = a.seg[0].ldy;
    const int64_t r0 = static_cast<int64_t>(grp) * 16 + g;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int t = nt * 8 + 2 * tq + (c & 1);
        if (t < a.M) y[t * ldy + r0 + (c >> 1) * 8] = silu_mul<OT>(v[0][nt][c], v[1][nt][c]);
      }
    return;
  }
  const int s = seg_of(a, grp);
  OT* y = static_cast<OT*>(a.seg[s].y);
  const int64_t ldy = a.seg[s].ldy;
  const int64_t base = static_cast<int64_t>(grp - (s ? a.seg_end[s - 1] : 0)) * 32 + g;
#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int t = nt * 8 + 2 * tq + (c & 1);
        if (t < a.M) y[t * ldy + base + rt * 16 + (c >> 1) * 8] = Dt<OT>::from_f32(v[rt][nt][c]);
      }
}

template <typename OT, int RT, int NT, bool SEG>
__device__ __forceinline__ void store_out(const GemmArgs& a, int grp, const float (&v)[RT][NT][4], int g, int tq) {
  if constexpr (SEG) store_seg<OT, NT>(a, grp, v, g, tq);
  else store_group<OT, RT, NT>(a, grp, v, g, tq);
}

template <int RT, int NT>
__device__ __forceinline__ void zero_acc(float (&acc)[RT][NT][4]) {
#pragma unroll
  for (int rt = 0; rt < RT; ++rt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[rt][nt][0] = acc[rt][nt][1] = acc[rt][nt][2] = acc[rt][nt][3] = 0.f;
}

// Unit ranges use 32-bit arithmetic (the host guarantees total * grid < 2^31): the serial parts of
// the kernel must not pay for 64-bit division.
__device__ __forceinline__ int cta_begin(int c, int total, int grid) { return c * total / grid; }
// CTA whose slice contains unit p: the largest c with floor(c*total/grid) <= p.
__device__ __forceinline__ int cta_of(int p, int total, int grid) { return ((p + 1) * grid - 1) / total; }

// Combine the per-warp partials of the row groups this CTA touched: warp i handles the i-th group
// (lanes own their fragment positions); its contributing warps are the contiguous range holding the
// group's units. Groups shared with neighbouring CTAs go through the workspace (see below).
template <typename OT, int RT, int NT, int NW, bool SEG>
__device__ __forceinline__ void combine_cta(const GemmArgs& a, const float* slots, const int* s_wa, const int* s_wb,
                                            const int* s_fg, int A, int B, int cta, int warp, int lane, int g,
                                            int tq) {
  constexpr int E = RT * NT * 128;
  const int grid = gridDim.x, upg = a.upg;
  if (A >= B) return;
  const int gA = A / upg, gB = (B - 1) / upg;
  const int span = B - A;
  for (int grp = gA + warp; grp <= gB; grp += NW) {
    const int lo = max(grp * upg, A), hi = min((grp + 1) * upg, B);   // this CTA's units of grp
    const bool shared = grp * upg < A || (grp + 1) * upg > B;          // other CTAs hold the rest
    const int w_lo = ((lo - A + 1) * NW - 1) / span, w_hi = ((hi - 1 - A + 1) * NW - 1) / span;
    if (!shared && w_lo == w_hi) continue;                            // one warp stored it in full
    float v[RT][NT][4];
    zero_acc(v);
    for (int w = w_lo; w <= w_hi; ++w) {
      if (s_wa[w] >= s_wb[w]) continue;   // a warp without units (CTA slice shorter than NW)
      const float* s = slots + (w * 2 + (grp == s_fg[w] ? 0 : 1)) * E + lane * 4;
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float4 q = *reinterpret_cast<const float4*>(s + (rt * NT + nt) * 128);
          v[rt][nt][0] += q.x; v[rt][nt][1] += q.y; v[rt][nt][2] += q.z; v[rt][nt][3] += q.w;
        }
    }
    if (!shared) {
      store_out<OT, RT, NT, SEG>(a, grp, v, g, tq);
      continue;
    }
    // Shared with neighbouring CTAs: publish this CTA's partial; the last arriver adds all partials
    // in CTA order. The lanes' stores are ordered before lane 0's release by the warp barrier; lane
    // 0's acquire (and the barrier after it) orders the last arriver's reads after every partial.
    float* mine = a.partials + (static_cast<int64_t>(cta) * 2 + (grp == gA ? 0 : 1)) * E + lane * 4;
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        __stcg(reinterpret_cast<float4*>(mine + (rt * NT + nt) * 128),
               make_float4(v[rt][nt][0], v[rt][nt][1], v[rt][nt][2], v[rt][nt][3]));
    __syncwarp();
    const int c_lo = cta_of(grp * upg, a.total, grid), c_hi = cta_of((grp + 1) * upg - 1, a.total, grid);
    int last = 0;
    if (lane == 0 && atomic_add_acq_rel_gpu(a.counters + grp, 1) == c_hi - c_lo) {
      last = 1;
      a.counters[grp] = 0;   // every contributor has arrived: reset for the next launch
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    __syncwarp();
    if (!last) continue;
    zero_acc(v);
    for (int c = c_lo; c <= c_hi; ++c) {
      const int cfirst = cta_begin(c, a.total, grid) / upg;
      const float* s = a.partials + (static_cast<int64_t>(c) * 2 + (grp == cfirst ? 0 : 1)) * E + lane * 4;
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float4 q = __ldcg(reinterpret_cast<const float4*>(s + (rt * NT + nt) * 128));
          v[rt][nt][0] += q.x; v[rt][nt][1] += q.y; v[rt][nt][2] += q.z; v[rt][nt][3] += q.w;
        }
    }
    store_out<OT, RT, NT, SEG>(a, grp, v, g, tq);
  }
}

template <typename T, typename OT, int RT, int NT, int CB, bool NESTED, int NW>
__global__ void __launch_bounds__(NW * 32, 1) nf4_gemm_tc_kernel(const GemmArgs a) {
  constexpr int E = RT * NT * 128;  // fp32 values of one group partial, in fragment order
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint8_t* lut = smem;
  float* code2_s = reinterpret_cast<float*>(smem + kLutBytes);
  float* slots = code2_s + 256;  // [warps][2][E]
  __shared__ int s_wa[NW], s_wb[NW], s_fg[NW];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const uint32_t lane4 = static_cast<uint32_t>(lane) * 4u;

  const int grid = gridDim.x, cta = blockIdx.x;
  const int A = cta_begin(cta, a.total, grid), B = cta_begin(cta + 1, a.total, grid);
  const int wa = A + warp * (B - A) / NW;
  const int wb = A + (warp + 1) * (B - A) / NW;
  const int upg = a.upg;
  const int first_grp = wa / upg;
  if (lane == 0) {
    s_wa[warp] = wa;
    s_wb[warp] = wb;
    s_fg[warp] = first_grp;
  }

  // table inputs first, then the first unit's weights, all in flight while the table is built
  const float my_code = __ldg(a.w.code + (lane & 15));
  float my_code2 = 0.f;
  if (NESTED && tid < 256) my_code2 = __ldg(a.w.code2 + tid);
  WBuf<RT, NT, CB, NESTED> buf0, buf1;
  int lgrp = first_grp;
  int lun = wa - lgrp * upg;
  if (wa < wb) load_w<T, RT, NT, CB, NESTED>(buf0, a, lgrp, lun, g, tq);
  if (++lun == upg) { lun = 0; ++lgrp; }

  // Warps 0..7 build the table: lane l of warp w computes entry e = 32w + l once and writes its 32
  // lane copies in a lane-rotated order, so every store instruction hits 32 distinct banks.
  {
    const int e = warp * 32 + lane;
    const float hi = __shfl_sync(0xffffffffu, my_code, (e >> 4) & 15);
    const float lo = __shfl_sync(0xffffffffu, my_code, e & 15);
    if (warp < 8) {
      const uint32_t val = Dt<T>::pack2(hi, lo);
      uint32_t* entry = reinterpret_cast<uint32_t*>(smem + e * kLutEntryBytes);
#pragma unroll
      for (int i = 0; i < 32; ++i) entry[(i + lane) & 31] = val;
    }
  }
  if (NESTED && tid < 256) code2_s[tid] = my_code2;
  __syncthreads();

  if (wa < wb) {
    float acc[RT][NT][4];
    zero_acc(acc);
    int cgrp = first_grp;
    int cun = wa - cgrp * upg;

    auto flush = [&](int grp) {
      const bool full = grp * upg >= wa && (grp + 1) * upg <= wb;
      if (full) {
        store_group<OT, RT, NT>(a, grp, acc, g, tq);
      } else {
        float* s = slots + (warp * 2 + (grp == first_grp ? 0 : 1)) * E + lane * 4;
#pragma unroll
        for (int rt = 0; rt < RT; ++rt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            *reinterpret_cast<float4*>(s + (rt * NT + nt) * 128) =
                make_float4(acc[rt][nt][0], acc[rt][nt][1], acc[rt][nt][2], acc[rt][nt][3]);
      }
      zero_acc(acc);
    };
    auto step = [&](WBuf<RT, NT, CB, NESTED>& cur, WBuf<RT, NT, CB, NESTED>& nxt, int p) {
      if (p + 1 < wb) {
        load_w<T, RT, NT, CB, NESTED>(nxt, a, lgrp, lun, g, tq);
        if (++lun == upg) { lun = 0; ++lgrp; }
      }
      compute_unit<T, RT, NT, CB, NESTED>(cur, a, cun, acc, lut, lane4, code2_s, g, tq);
      if (++cun == upg) {
        flush(cgrp);
        cun = 0;
        ++cgrp;
      }
    };
    for (int p = wa; p < wb; p += 2) {
      step(buf0, buf1, p);
      if (p + 1 < wb) step(buf1, buf0, p + 1);
    }
    if (cun != 0) flush(cgrp);  // range ended inside a group
  }
  __syncthreads();

  combine_cta<OT, RT, NT, NW, false>(a, slots, s_wa, s_wb, s_fg, A, B, cta, warp, lane, g, tq);
}

// ------------------------------------------------------------------------------------------
// Pipelined variant for 32-row groups and 4-block units (the common M <= 8 decode shapes): each warp
// streams its units through a private ring of R shared-memory stages filled by 16-byte cp.async
// copies (8 lanes per 128-byte row segment, so one copy instruction moves 4 whole rows), with the
// per-row scales riding in the same stage. R-1 units per warp are in flight while one is computed,
// and no registers hold them; the activations of the next unit (all 4 blocks) are loaded into
// registers while the current one is computed. Inside a stage, the 16-byte chunk c of row r sits at
// chunk c ^ 2*(r & 3): the fragment reads (8 bytes per lane, 4 rows x 2 chunks per half-warp) then
// hit 32 distinct banks without padding.
//
// The kernel also serves segmented launches: several weights that share x (q/k/v, or gate/up)
// in one launch, their row groups concatenated. In paired mode a 32-row group is 16 rows of
// segment 0 (tile 0) and the same 16 rows of segment 1 (tile 1), and the epilogue writes
// silu(seg0 . x) * (seg1 . x) with the rounding of the model dtype (the SwiGLU of a Mistral MLP).
constexpr int kStageW = 32 * 128;                // weights of one unit: 32 rows x 4 blocks x 32 B
constexpr int kStageBytes = kStageW + 32 * 16;   // + scales, 16 B per row

__device__ __forceinline__ int swz(int r, int c) { return r * 128 + ((c ^ (2 * (r & 3))) << 4); }

// Rows 0..15 and 16..31 of group grp: their segments and the segment-local index of their first row.
__device__ __forceinline__ void halves_of(const GemmArgs& a, int grp, int& s_lo, int& s_hi, int64_t& r_lo,
                                          int64_t& r_hi) {
  if (a.pair) {
    s_lo = 0; s_hi = 1;
    r_lo = r_hi = static_cast<int64_t>(grp) * 16;
  } else {
    s_lo = s_hi = seg_of(a, grp);
    r_lo = static_cast<int64_t>(grp - (s_lo ? a.seg_end[s_lo - 1] : 0)) * 32;
    r_hi = r_lo + 16;
  }
}

// A lane's copy sources for the units of one group: its weight chunk (16 bytes) of rows rr and
// 16 + rr (rr = lane / 8; rows 4i further are 4i row strides on), and the scales of row `lane`.
struct IssueCursor {
  const uint8_t* pl;
  const uint8_t* ph;
  int64_t sl, sh;        // 4-row strides in bytes
  const uint8_t* sa;     // the row's absmax at unit 0 (bytes)
  const float* a2;       // absmax2 (double quant)
  int64_t gb;            // the row's first block in the full tensor (double quant)
};

template <bool NESTED>
__device__ __forceinline__ IssueCursor cursor_for(const GemmArgs& a, int grp, int lane) {
  int s_lo, s_hi;
  int64_t r_lo, r_hi;
  halves_of(a, grp, s_lo, s_hi, r_lo, r_hi);
  const int c = lane & 7, rr = lane >> 3;
  const Nf4View& wl = a.seg[s_lo].w;
  const Nf4View& wh = a.seg[s_hi].w;
  IssueCursor k;
  k.pl = wl.packed + (r_lo + rr) * wl.ld_packed + c * 16;
  k.ph = wh.packed + (r_hi + rr) * wh.ld_packed + c * 16;
  k.sl = 4 * wl.ld_packed;
  k.sh = 4 * wh.ld_packed;
  const bool hi = lane >= 16;
  const Nf4View& w = hi ? wh : wl;
  const int64_t row = (hi ? r_hi : r_lo) + (lane & 15);
  k.sa = static_cast<const uint8_t*>(w.absmax) + row * w.ld_absmax * (NESTED ? 1 : 4);
  k.a2 = w.absmax2;
  k.gb = w.gblk_base + row * w.gblk_row_stride;
  return k;
}

// Copy one unit (32 rows x 4 blocks + the rows' scales) into stage st. wdst = this lane's chunk slot
// for row rr (rows 4i on are 512*i bytes further: the swizzle depends on r & 3 only).
template <bool NESTED>
__device__ __forceinline__ void issue_unit(uint32_t st, const IssueCursor& k, int unit, uint32_t wdst, int lane) {
  const int64_t uo = static_cast<int64_t>(unit) * 128;
#pragma unroll
  for (int i = 0; i < 4; ++i) cp_async16(st + wdst + 512 * i, k.pl + uo + i * k.sl);
#pragma unroll
  for (int i = 0; i < 4; ++i) cp_async16(st + wdst + 2048 + 512 * i, k.ph + uo + i * k.sh);
  const uint32_t sdst = st + kStageW + lane * 16;
  if (NESTED) {
    // a unit never straddles a 256-block group of absmax2 (the host guarantees 4-alignment)
    cp_async4(sdst, k.sa + unit * 4);
    cp_async4(sdst + 4, k.a2 + ((k.gb + unit * 4) >> 8));
  } else {
    cp_async16(sdst, k.sa + unit * 16);
  }
}

// Activations of one unit (4 blocks). xrow[nt] is the lane's row of x for token nt*8 + g, clamped to
// a valid row: lanes past M read real data whose MMA output columns are never stored, so the loads
// need neither a branch nor zeroing.
template <typename T, int NT>
__device__ __forceinline__ void load_x_unit(uint4 (&xv)[4][NT][2], const T* const (&xrow)[NT], int unit) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const T* p = xrow[nt] + (unit * 4 + j) * 64;
      xv[j][nt][0] = ldg_u4(p);
      xv[j][nt][1] = ldg_u4(p + 8);
    }
}

// Lane L turns row L's raw double-quantised scales (4 code2 indices + the group's absmax2) into the
// 4 fp32 block scales, in place in the stage.
__device__ __forceinline__ void decode_scales(uint8_t* stage, const float* c2, float off, int lane) {
  uint8_t* sp = stage + kStageW + lane * 16;
  const uint32_t q4 = *reinterpret_cast<const uint32_t*>(sp);
  const float a2 = *reinterpret_cast<const float*>(sp + 4);
  float4 v;
  v.x = __fadd_rn(__fmul_rn(c2[q4 & 0xFF], a2), off);
  v.y = __fadd_rn(__fmul_rn(c2[(q4 >> 8) & 0xFF], a2), off);
  v.z = __fadd_rn(__fmul_rn(c2[(q4 >> 16) & 0xFF], a2), off);
  v.w = __fadd_rn(__fmul_rn(c2[q4 >> 24], a2), off);
  *reinterpret_cast<float4*>(sp) = v;
}

// One staged unit for a warp: 2 row tiles x 4 blocks; xv = the unit's activations. The lane's
// fragment bytes of block j, row rt*16 + h*8 + g sit at wb + (rt*16 + h*8)*128 + jx[j] (the stage
// swizzle: chunk c of row r at c ^ 2(r & 3), and r & 3 == g & 3 for all four rows).
template <typename T, int NT>
__device__ __forceinline__ void compute_staged(const uint8_t* stage, const uint8_t* wb, const int (&jx)[4],
                                               const uint4 (&xv)[4][NT][2], float (&acc)[2][NT][4],
                                               const uint8_t* lut, uint32_t lane4, int g) {
  float sc[2][2][4];
#pragma unroll
  for (int rt = 0; rt < 2; ++rt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float4 v = *reinterpret_cast<const float4*>(stage + kStageW + (rt * 16 + h * 8 + g) * 16);
      sc[rt][h][0] = v.x; sc[rt][h][1] = v.y; sc[rt][h][2] = v.z; sc[rt][h][3] = v.w;
    }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int rt = 0; rt < 2; ++rt) {
      const uint2 wg = *reinterpret_cast<const uint2*>(wb + jx[j] + rt * 2048);
      const uint2 wh = *reinterpret_cast<const uint2*>(wb + jx[j] + rt * 2048 + 1024);
      float c[NT][4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const uint32_t w0 = (s < 2) ? wg.x : wg.y;
        const uint32_t w1 = (s < 2) ? wh.x : wh.y;
        const uint32_t sel0 = (s & 1) ? 0x5524u : 0x5504u;
        const uint32_t sel1 = (s & 1) ? 0x5534u : 0x5514u;
        const uint32_t a0 = lut_lookup(lut, w0, lane4, sel0);
        const uint32_t a2 = lut_lookup(lut, w0, lane4, sel1);
        const uint32_t a1 = lut_lookup(lut, w1, lane4, sel0);
        const uint32_t a3 = lut_lookup(lut, w1, lane4, sel1);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv[j][nt][0]);
          if (s == 0) Mma<T>::run0(c[nt], a0, a1, a2, a3, xw[0], xw[1]);
          else Mma<T>::run(c[nt], a0, a1, a2, a3, xw[2 * s], xw[2 * s + 1]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        acc[rt][nt][0] = fmaf(sc[rt][0][j], c[nt][0], acc[rt][nt][0]);
        acc[rt][nt][1] = fmaf(sc[rt][0][j], c[nt][1], acc[rt][nt][1]);
        acc[rt][nt][2] = fmaf(sc[rt][1][j], c[nt][2], acc[rt][nt][2]);
        acc[rt][nt][3] = fmaf(sc[rt][1][j], c[nt][3], acc[rt][nt][3]);
      }
    }
  }
}

template <int NW, int R, int NT>
constexpr size_t pipe_smem_bytes() {
  return kLutBytes + kMaxSeg * kCode2Bytes + static_cast<size_t>(NW + 1) * 2 * (2 * NT * 128) * 4 +
         static_cast<size_t>(NW) * R * kStageBytes;
}

// Combine for the cluster partition: a CTA sums its warps' parts of every group it touched; a group
// held by one CTA is stored at once, a group split between CTAs of the cluster is left in part[] and,
// after a cluster barrier, the first CTA holding it adds the others' parts (distributed shared
// memory, in rank order) and stores it. A second barrier keeps every CTA's part[] alive until read.
template <typename OT, int NT, int NW, int EPI>
__device__ __forceinline__ void combine_cluster(const GemmArgs& a, const float* slots, float* part, const int* s_wa,
                                                const int* s_wb, const int* s_fg, int A, int B, int U0, int n,
                                                int q, int cs, int warp, int lane, int g, int tq, uint32_t epoch) {
  constexpr int E = 2 * NT * 128;
  const int upg = a.upg;
  const int gA = A / upg, gB = B > A ? (B - 1) / upg : gA - 1;
  const int span = B - A;
  for (int grp = gA + warp; grp <= gB; grp += NW) {
    const int lo = max(grp * upg, A), hi = min((grp + 1) * upg, B);
    const bool shared = grp * upg < A || (grp + 1) * upg > B;
    const int w_lo = ((lo - A + 1) * NW - 1) / span, w_hi = ((hi - 1 - A + 1) * NW - 1) / span;
    if (!shared && w_lo == w_hi) continue;   // one warp stored it in full
    float v[2][NT][4];
    zero_acc(v);
    for (int w = w_lo; w <= w_hi; ++w) {
      if (s_wa[w] >= s_wb[w]) continue;
      const float* s = slots + (w * 2 + (grp == s_fg[w] ? 0 : 1)) * E + lane * 4;
#pragma unroll
      for (int rt = 0; rt < 2; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float4 t = *reinterpret_cast<const float4*>(s + (rt * NT + nt) * 128);
          v[rt][nt][0] += t.x; v[rt][nt][1] += t.y; v[rt][nt][2] += t.z; v[rt][nt][3] += t.w;
        }
    }
    if (!shared) {
      store_seg<OT, NT, EPI>(a, grp, v, g, tq, epoch);
      continue;
    }
    float* d = part + (grp == gA ? 0 : 1) * E + lane * 4;
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        *reinterpret_cast<float4*>(d + (rt * NT + nt) * 128) =
            make_float4(v[rt][nt][0], v[rt][nt][1], v[rt][nt][2], v[rt][nt][3]);
  }
  if (cs == 1) return;   // a lone CTA holds its groups whole: nothing is shared, no cluster barrier
  cluster_sync();
  // owners: warp 0 takes the CTA's first group, warp 1 its last (when shared and first held here)
  if (warp < 2 && span > 0) {
    const int grp = warp == 0 ? gA : gB;
    const bool shared = grp * upg < A || (grp + 1) * upg > B;
    const int q_lo = ((grp * upg - U0 + 1) * cs - 1) / n;
    if (shared && q_lo == q && !(warp == 1 && gB == gA)) {
      const int q_hi = (((grp + 1) * upg - 1 - U0 + 1) * cs - 1) / n;
      float v[2][NT][4];
      const float* mine = part + (grp == gA ? 0 : 1) * E + lane * 4;
#pragma unroll
      for (int rt = 0; rt < 2; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float4 t = *reinterpret_cast<const float4*>(mine + (rt * NT + nt) * 128);
          v[rt][nt][0] = t.x; v[rt][nt][1] = t.y; v[rt][nt][2] = t.z; v[rt][nt][3] = t.w;
        }
      for (int r = q + 1; r <= q_hi; ++r) {
        if (r * n / cs == (r + 1) * n / cs) continue;   // a rank without units (fewer units than CTAs)
        const int r_first = (U0 + r * n / cs) / upg;   // rank r's first group
        const uint32_t la = smem_u32(part + (grp == r_first ? 0 : 1) * E + lane * 4);
#pragma unroll
        for (int rt = 0; rt < 2; ++rt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const float4 t = ld_dsmem_f4(la + (rt * NT + nt) * 512, r);
            v[rt][nt][0] += t.x; v[rt][nt][1] += t.y; v[rt][nt][2] += t.z; v[rt][nt][3] += t.w;
          }
      }
      store_seg<OT, NT, EPI>(a, grp, v, g, tq, epoch);
    }
  }
  // keeps this CTA's part[] alive until the owners have read it; their loaded values are consumed
  // (stored) before they arrive, so the barrier needs no memory ordering
  cluster_sync_relaxed();
}

template <typename T, typename OT, int NT, bool NESTED, int NW, int R, int EPI>
__global__ void __launch_bounds__(NW * 32, 1) nf4_gemm_pipe_kernel(const GemmArgs a) {
  constexpr int RT = 2;
  constexpr int E = RT * NT * 128;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint8_t* lut = smem;
  float* code2_s = reinterpret_cast<float*>(smem + kLutBytes);        // [kMaxSeg][256]
  float* slots = code2_s + kMaxSeg * 256;                             // [NW][2][E]
  float* part = slots + NW * 2 * E;                                   // [2][E] cluster-shared groups
  uint8_t* rings = reinterpret_cast<uint8_t*>(part + 2 * E);         // [NW][R][kStageBytes]
  __shared__ int s_wa[NW], s_wb[NW], s_fg[NW];

  pdl_launch_dependents();   // the next kernel in the stream may start its own prologue
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const uint32_t lane4 = static_cast<uint32_t>(lane) * 4u;
  // Cluster partition: cluster c owns row groups [c*G/ncl, (c+1)*G/ncl) whole; its units (group-major)
  // are split evenly over its cs CTAs, so K is split only inside a cluster (32-bit math: the host
  // keeps G*ncl and units*cs below 2^31).
  const int cs = cluster_size(), q = cluster_rank(), cl = cluster_index(), ncl = cluster_count();
  const int upg0 = a.upg;
  const int grp0 = cl * a.groups / ncl, grp1 = (cl + 1) * a.groups / ncl;
  const int U0 = grp0 * upg0, n_cl = (grp1 - grp0) * upg0;
  const int A = U0 + q * n_cl / cs, B = U0 + (q + 1) * n_cl / cs;
  const int wa = A + warp * (B - A) / NW, wb = A + (warp + 1) * (B - A) / NW;
  const int upg = a.upg;
  const int first_grp = wa / upg;
  if (lane == 0) { s_wa[warp] = wa; s_wb[warp] = wb; s_fg[warp] = first_grp; }

  uint8_t* ring = rings + warp * (R * kStageBytes);
  const uint32_t ring_s = smem_u32(ring);
  const uint32_t wdst = swz(lane >> 3, lane & 7);
  if (!a.static_w) pdl_wait();   // weights may be the preceding kernel's output
  const float my_code = a.code_by_value ? a.code_v[lane & 15] : __ldg(a.seg[0].w.code + (lane & 15));
  // The first R-1 units (and the code2 tables, with group 0) are in flight while the dequant table
  // is built.
  if (NESTED)
    for (int i = tid; i < a.nseg * 256; i += NW * 32) cp_async4(smem_u32(code2_s + i), a.seg[i >> 8].w.code2 + (i & 255));
  int igrp = first_grp, iun = wa - first_grp * upg;
  IssueCursor cur = cursor_for<NESTED>(a, igrp, lane);
#pragma unroll
  for (int s = 0; s < R - 1; ++s) {
    if (wa + s < wb) {
      issue_unit<NESTED>(ring_s + s * kStageBytes, cur, iun, wdst, lane);
      if (++iun == upg) {
        iun = 0;
        ++igrp;
        if (wa + s + 1 < wb) cur = cursor_for<NESTED>(a, igrp, lane);
      }
    }
    cp_async_commit();
  }
  // table build: lane l of pass w computes entry 32w + l once and writes its 32 lane copies in a
  // lane-rotated order, so every store instruction hits 32 distinct banks
  for (int ew = warp; ew < 8; ew += NW) {
    const int e = ew * 32 + lane;
    const float hi = __shfl_sync(0xffffffffu, my_code, (e >> 4) & 15);
    const float lo = __shfl_sync(0xffffffffu, my_code, e & 15);
    const uint32_t val = Dt<T>::pack2(hi, lo);
    uint32_t* entry = reinterpret_cast<uint32_t*>(smem + e * kLutEntryBytes);
#pragma unroll
    for (int i = 0; i < 32; ++i) entry[(i + lane) & 31] = val;
  }
  if (NESTED) cp_async_wait<R - 2>();   // this thread's code2 copies (group 0) have landed
  __syncthreads();
  pdl_wait();   // x, the workspace and the outputs belong to the stream order from here on
  const uint32_t epoch = EPI == kEpiAllReduce ? ar_epoch(a.are) : 0u;

  if (wa < wb) {
    float acc[RT][NT][4];
    zero_acc(acc);
    int cgrp = first_grp, cun = wa - first_grp * upg;
    int st_c = 0, st_i = R - 1;   // stages of the unit computed / issued next
    const uint8_t* wbase0 = ring + g * 128 + 8 * tq;
    int jx[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) jx[j] = (j ^ (g & 3)) << 5;
    const int c2_lane_seg = lane >> 4;
    const T* xrow[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int tok = nt * 8 + g < a.M ? nt * 8 + g : 0;
      xrow[nt] = static_cast<const T*>(a.x) + tok * a.ldx + tq * 16;
    }
    uint4 xa[4][NT][2], xb[4][NT][2];
    load_x_unit<T, NT>(xa, xrow, cun);
    auto park = [&](int grp) {   // a group this warp holds only part of: leave it for the combine
      float* s = slots + (warp * 2 + (grp == first_grp ? 0 : 1)) * E + lane * 4;
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          *reinterpret_cast<float4*>(s + (rt * NT + nt) * 128) =
              make_float4(acc[rt][nt][0], acc[rt][nt][1], acc[rt][nt][2], acc[rt][nt][3]);
    };
    // scale-decode table and offset of the group being computed (lane's row segment in paired mode)
    int dseg = a.pair ? c2_lane_seg : seg_of(a, cgrp);
    const float* dtab = code2_s + dseg * 256;
    float doff = a.seg[dseg].w.offset;
    auto step = [&](const uint4 (&xc)[4][NT][2], uint4 (&xn)[4][NT][2], int p) {
      if (p + R - 1 < wb) {
        issue_unit<NESTED>(ring_s + st_i * kStageBytes, cur, iun, wdst, lane);
        if (++iun == upg) {
          iun = 0;
          ++igrp;
          if (p + R < wb) cur = cursor_for<NESTED>(a, igrp, lane);   // the next issue opens this group
        }
      }
      st_i = st_i + 1 == R ? 0 : st_i + 1;
      cp_async_commit();
      if (p + 1 < wb) load_x_unit<T, NT>(xn, xrow, cun + 1 < upg ? cun + 1 : 0);   // may open a new group
      cp_async_wait<R - 1>();
      __syncwarp();
      uint8_t* stage = ring + st_c * kStageBytes;
      if (NESTED) {
        decode_scales(stage, dtab, doff, lane);
        __syncwarp();
      }
      compute_staged<T, NT>(stage, wbase0 + st_c * kStageBytes, jx, xc, acc, lut, lane4, g);
      __syncwarp();   // every lane is done with the stage before it is refilled
      st_c = st_c + 1 == R ? 0 : st_c + 1;
      if (++cun == upg) {
        if (cgrp * upg >= wa) store_seg<OT, NT, EPI>(a, cgrp, acc, g, tq, epoch);
        else park(cgrp);
        zero_acc(acc);
        cun = 0;
        ++cgrp;
        if (NESTED && !a.pair && p + 1 < wb) {
          dseg = seg_of(a, cgrp);
          dtab = code2_s + dseg * 256;
          doff = a.seg[dseg].w.offset;
        }
      }
    };
    for (int p = wa; p < wb; p += 2) {
      step(xa, xb, p);
      if (p + 1 < wb) step(xb, xa, p + 1);
    }
    if (cun != 0) park(cgrp);   // range ended inside a group
  }
  cp_async_wait<0>();
  __syncthreads();
  combine_cluster<OT, NT, NW, EPI>(a, slots, part, s_wa, s_wb, s_fg, A, B, U0, n_cl, q, cs, warp, lane, g, tq, epoch);
}

// ------------------------------------------------------------------------------------------
// CUDA-core comparison kernel (M <= 8): one warp per output row at a time, lane l covers 32
// consecutive weights (half a block) of every 1024-weight segment, fp32 FMAs against fp32 code
// values scaled once per block, one warp-shuffle reduction per token per row.
constexpr int kSimtThreads = 256;

template <typename T, typename OT, int MT, bool NESTED>
__global__ void __launch_bounds__(kSimtThreads) nf4_gemv_simt_kernel(const GemmArgs a) {
  __shared__ float code_s[16 * 32];
  __shared__ float code2_s[256];
  const int tid = threadIdx.x, lane = tid & 31;
  for (int i = tid; i < 16 * 32; i += kSimtThreads) code_s[i] = __ldg(a.w.code + (i >> 5));
  if (NESTED)
    for (int i = tid; i < 256; i += kSimtThreads) code2_s[i] = __ldg(a.w.code2 + i);
  __syncthreads();
  const T* x = static_cast<const T*>(a.x);
  OT* y = static_cast<OT*>(a.y);
  const int warps_total = gridDim.x * (kSimtThreads / 32);
  const int gw = blockIdx.x * (kSimtThreads / 32) + (tid >> 5);
  for (int64_t row = gw; row < a.N; row += warps_total) {
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.f;
    for (int k0 = lane * 32; k0 < a.K; k0 += 32 * 32) {
      const int blk = k0 >> 6;
      const uint4 wv = ldg_stream_u4(a.w.packed + row * a.w.ld_packed + (k0 >> 1));
      float sc;
      const int64_t bi = row * a.w.ld_absmax + blk;
      if (NESTED) {
        const int64_t gb = a.w.gblk_base + row * a.w.gblk_row_stride + blk;
        sc = __fadd_rn(__fmul_rn(code2_s[__ldg(static_cast<const uint8_t*>(a.w.absmax) + bi)],
                                 __ldg(a.w.absmax2 + (gb >> 8))), a.w.offset);
      } else {
        sc = __ldg(static_cast<const float*>(a.w.absmax) + bi);
      }
      const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
      float part[MT];
#pragma unroll
      for (int m = 0; m < MT; ++m) part[m] = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float wf[8];
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
          const uint32_t byte = byte_of(ws[q], bb);
          wf[2 * bb] = code_s[((byte >> 4) << 5) + lane];
          wf[2 * bb + 1] = code_s[((byte & 15u) << 5) + lane];
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m < a.M) {
            const uint4 xv = ldg_u4(x + m * a.ldx + k0 + q * 8);
            const T* xh = reinterpret_cast<const T*>(&xv);
#pragma unroll
            for (int e = 0; e < 8; ++e) part[m] = fmaf(wf[e], Dt<T>::to_f32(xh[e]), part[m]);
          }
        }
      }
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[m] = fmaf(sc, part[m], acc[m]);
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float v = acc[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && m < a.M) y[m * a.ldy + row] = Dt<OT>::from_f32(v);
    }
  }
}

// ------------------------------------------------------------------------------------------ host

// Workspace layout: a fixed-size counter region first (so calls of any shape agree on where the
// counters live and always find them zero), then the per-CTA partial slots.
constexpr size_t kCounterBytes = 64 * 1024;
constexpr size_t kErrWordOffset = kCounterBytes - 64;   // the TMA-staged kernel's timeout counter
constexpr int64_t kMaxGroups = kErrWordOffset / 4;

// Which M <= 8 kernel serves a launch: the register-staged one (default: measured faster on B200, in
// isolation and inside the decode step), or, with B2D_NF4_KERNEL=tma in the environment, the TMA-staged
// one when its rules are met (read at every call: a comparison can switch between calls).
bool tma_path_enabled() {
  const char* v = std::getenv("B2D_NF4_KERNEL");
  return v && std::strcmp(v, "tma") == 0;
}

// 9..64 tokens run the tcgen05 kernel (nf4_tc5.cu) when its rules are met; B2D_NF4_TC5=0 in the
// environment selects the register-staged mma.sync kernel instead (read at every call, for comparisons).
bool tc5_path_enabled() {
  const char* v = std::getenv("B2D_NF4_TC5");
  return !(v && std::strcmp(v, "0") == 0);
}

Nf4TmaSegment tma_segment(const uint8_t* packed, int64_t ld_packed, const void* absmax, int64_t ld_absmax,
                          const float* code2, const float* absmax2, float offset, int64_t gblk_base,
                          int64_t gblk_row_stride, int N, void* y, int64_t ldy) {
  Nf4TmaSegment t;
  t.packed = packed; t.ld_packed = ld_packed;
  t.absmax = absmax; t.ld_absmax = ld_absmax;
  t.code2 = code2; t.absmax2 = absmax2; t.offset = offset;
  t.gblk_base = gblk_base; t.gblk_row_stride = gblk_row_stride;
  t.N = N; t.y = y; t.ldy = ldy;
  return t;
}

struct GemmConfig {
  int rt, nt, cb, nw;
  int64_t groups, total;
  int grid;
  size_t counter_bytes, partial_bytes;
};

bool chunk4_ok(int K, const void* absmax, int64_t ld_absmax, int nested, int64_t gblk_base, int64_t gblk_row_stride) {
  if ((K / 64) % 4 != 0 || ld_absmax % 4 != 0) return false;
  if (nested) return aligned(absmax, 4) && gblk_base % 4 == 0 && gblk_row_stride % 4 == 0;
  return aligned(absmax, 16);
}

int choose_config(int M, int N, int K, bool chunk4, const DeviceInfo& di, GemmConfig* c) {
  c->nt = M <= 8 ? 1 : (M <= 16 ? 2 : (M <= 32 ? 4 : 8));
  c->rt = (c->nt == 1 && N % 32 == 0) ? 2 : 1;
  c->cb = chunk4 ? 4 : 1;
  c->nw = c->nt > 2 ? 8 : (c->nt == 2 ? 12 : (c->rt == 2 ? 10 : 16));
  c->groups = N / (16 * c->rt);
  c->total = c->groups * (K / (64 * c->cb));
  int64_t grid = di.sm_count;
  if (grid > c->total) grid = c->total;
  if (grid < 1) grid = 1;
  c->grid = static_cast<int>(grid);
  c->counter_bytes = kCounterBytes;
  c->partial_bytes = static_cast<size_t>(c->grid) * 2 * (c->rt * c->nt * 128) * 4;
  if (c->groups > kMaxGroups || c->total * static_cast<int64_t>(c->grid) >= (int64_t(1) << 31)) return B2D_ERR_SHAPE;
  return B2D_OK;
}

size_t gemm_smem_bytes(int rt, int nt, int nw) {
  return kLutBytes + kCode2Bytes + static_cast<size_t>(nw) * 2 * rt * nt * 128 * 4;
}

template <typename T, typename OT, int RT, int NT, int CB, bool NESTED, int NW>
int launch_tc(const GemmArgs& a, int grid, cudaStream_t stream) {
  auto kern = nf4_gemm_tc_kernel<T, OT, RT, NT, CB, NESTED, NW>;
  const size_t smem = gemm_smem_bytes(RT, NT, NW);
  static bool configured[64] = {false};   // per device; setting it twice is harmless
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return B2D_ERR_DEVICE;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) { set_cuda_error(e); return B2D_ERR_LAUNCH; }
    configured[dev] = true;
  }
  kern<<<grid, NW * 32, smem, stream>>>(a);
  return launch_status();
}

#ifndef B2D_PIPE_NW
#define B2D_PIPE_NW 8   // warps of the pipelined kernel
#endif
#ifndef B2D_PIPE_RING
#define B2D_PIPE_RING 3   // stages per warp
#endif

// Cluster size for the pipelined kernel: K is split only inside a cluster, whose CTAs own whole row
// groups, so the choice trades load balance (groups per cluster) against the cluster reduction.
// Picks the size with the fewest units per CTA on the slowest cluster; ties go to the smaller size.
struct PipeLaunch {
  int cs, ncl;
};

template <typename T, typename OT, bool NESTED, int NW, int R, int EPI>
int launch_pipe(const GemmArgs& a, bool pdl, cudaStream_t stream) {
  auto kern = nf4_gemm_pipe_kernel<T, OT, 1, NESTED, NW, R, EPI>;
  constexpr size_t smem = pipe_smem_bytes<NW, R, 1>();
  constexpr int kSizes[4] = {1, 2, 4, 8};
  static int max_clusters[64][4] = {};   // per device and size; 0 = not queried yet, -1 = unavailable
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return B2D_ERR_DEVICE;
  if (max_clusters[dev][0] == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) { set_cuda_error(e); return B2D_ERR_LAUNCH; }
    DeviceInfo di;
    if (device_info(&di) != B2D_OK) return B2D_ERR_DEVICE;
    for (int i = 0; i < 4; ++i) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(kSizes[i] * (di.sm_count / kSizes[i]));
      cfg.blockDim = dim3(NW * 32);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = kSizes[i];
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int m = 0;
      if (cudaOccupancyMaxActiveClusters(&m, kern, &cfg) != cudaSuccess || m <= 0) {
        cudaGetLastError();
        m = i == 0 ? di.sm_count : -1;
      }
      max_clusters[dev][i] = m;
    }
  }
  PipeLaunch best{1, 0};
  int64_t best_cost = -1;
  for (int i = 0; i < 4; ++i) {
    const int m = max_clusters[dev][i];
    if (m <= 0) continue;
    const int ncl = m < a.groups ? m : a.groups;
    const int64_t per_cluster = (static_cast<int64_t>(a.groups) + ncl - 1) / ncl * a.upg;
    const int64_t cost = (per_cluster + kSizes[i] - 1) / kSizes[i];   // units on the busiest CTA
    if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = PipeLaunch{kSizes[i], ncl}; }
  }
  if (best.ncl <= 0) return B2D_ERR_DEVICE;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(best.cs * best.ncl);
  cfg.blockDim = dim3(NW * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = best.cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) { set_cuda_error(e); return B2D_ERR_LAUNCH; }
  return launch_status();
}

template <typename T, typename OT, int EPI>
int dispatch_pipe_epi(const GemmArgs& a, int nested, bool pdl, cudaStream_t s) {
  return nested ? launch_pipe<T, OT, true, B2D_PIPE_NW, B2D_PIPE_RING, EPI>(a, pdl, s)
                : launch_pipe<T, OT, false, B2D_PIPE_NW, B2D_PIPE_RING, EPI>(a, pdl, s);
}

template <typename T, typename OT>
int dispatch_pipe(const GemmArgs& a, int nested, bool pdl, cudaStream_t s) {
  if (a.ar) {
    if constexpr (std::is_same<OT, float>::value) return B2D_ERR_DTYPE;
    else return dispatch_pipe_epi<T, OT, kEpiAllReduce>(a, nested, pdl, s);
  }
  return dispatch_pipe_epi<T, OT, kEpiStore>(a, nested, pdl, s);
}

template <typename T, typename OT, int CB, bool NESTED>
int dispatch_tc_cb(const GemmArgs& a, const GemmConfig& c, cudaStream_t s) {
#ifndef B2D_PIPE_OFF
  if (CB == 4 && c.nt == 1 && c.rt == 2)
    return launch_pipe<T, OT, NESTED, B2D_PIPE_NW, B2D_PIPE_RING, kEpiStore>(a, false, s);
#endif
  if (c.nt == 1)
    return c.rt == 2 ? launch_tc<T, OT, 2, 1, CB, NESTED, 10>(a, c.grid, s)
                     : launch_tc<T, OT, 1, 1, CB, NESTED, 16>(a, c.grid, s);
  if (c.nt == 2) return launch_tc<T, OT, 1, 2, CB, NESTED, 12>(a, c.grid, s);
  if (c.nt == 4) return launch_tc<T, OT, 1, 4, CB, NESTED, 8>(a, c.grid, s);
  return launch_tc<T, OT, 1, 8, CB, NESTED, 8>(a, c.grid, s);
}

template <typename T, typename OT>
int dispatch_tc(const GemmArgs& a, const GemmConfig& c, int nested, cudaStream_t s) {
  if (c.cb == 4)
    return nested ? dispatch_tc_cb<T, OT, 4, true>(a, c, s) : dispatch_tc_cb<T, OT, 4, false>(a, c, s);
  return nested ? dispatch_tc_cb<T, OT, 1, true>(a, c, s) : dispatch_tc_cb<T, OT, 1, false>(a, c, s);
}

int check_weight_args(const void* x, int64_t ldx, const uint8_t* packed, int64_t ld_packed, const void* absmax,
                      int64_t ld_absmax, int nested, const float* code2, const float* absmax2, const float* code,
                      const void* y, int64_t ldy, int M, int N, int K, int dtype, int y_dtype, int max_m) {
  if (M < 0 || N < 0 || K < 0) return B2D_ERR_ARG;
  if (dtype != B2D_F16 && dtype != B2D_BF16) return B2D_ERR_DTYPE;
  if (y_dtype != dtype && y_dtype != B2D_F32) return B2D_ERR_DTYPE;
  if (M > max_m || N % 16 != 0 || K % 64 != 0 || K == 0) return B2D_ERR_SHAPE;
  if (M == 0 || N == 0) return B2D_OK;
  if (!x || !packed || !absmax || !code || !y) return B2D_ERR_ARG;
  if (nested && (!code2 || !absmax2)) return B2D_ERR_ARG;
  if (ld_packed < K / 2 || ld_absmax < K / 64 || ldx < K || ldy < N) return B2D_ERR_SHAPE;
  if (!aligned(x, 16) || ldx % 8 != 0 || !aligned(packed, 16) || ld_packed % 16 != 0) return B2D_ERR_ALIGN;
  if (!nested && !aligned(absmax, 4)) return B2D_ERR_ALIGN;
  return B2D_OK;
}

}  // namespace

}  // namespace b2d

using namespace b2d;

extern "C" size_t b2d_nf4_gemm_workspace_bytes(int M, int N, int K) {
  DeviceInfo di;
  if (device_info(&di) != B2D_OK) return 0;
  if (M <= 0 || N <= 0 || K <= 0 || N % 16 || K % 64) return 0;
  GemmConfig c;
  // the 1-block chunking has the most units, hence the largest grid: size for it
  if (choose_config(M, N, K, false, di, &c) != B2D_OK) return 0;
  return c.counter_bytes + c.partial_bytes;
}

extern "C" int b2d_nf4_gemm(const void* x, int64_t ldx, const uint8_t* packed, int64_t ld_packed,
                            const void* absmax, int64_t ld_absmax, int nested, const float* code2,
                            const float* absmax2, float offset, int64_t gblk_base, int64_t gblk_row_stride,
                            const float* code, void* y, int64_t ldy, int M, int N, int K, int dtype,
                            int y_dtype, void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_weight_args(x, ldx, packed, ld_packed, absmax, ld_absmax, nested, code2, absmax2, code, y, ldy, M,
                             N, K, dtype, y_dtype, 64);
  if (st != B2D_OK || M == 0 || N == 0) return st;
  DeviceInfo di;
  if ((st = device_info(&di)) != B2D_OK) return st;
  GemmConfig c;
  const bool c4 = chunk4_ok(K, absmax, ld_absmax, nested, gblk_base, gblk_row_stride);
  if ((st = choose_config(M, N, K, c4, di, &c)) != B2D_OK) return st;
  if (!workspace || workspace_bytes < c.counter_bytes + c.partial_bytes) return B2D_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return B2D_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M <= 8 && tma_path_enabled()) {
    Nf4TmaLaunch L;
    std::memset(&L, 0, sizeof(L));
    L.x = x; L.ldx = ldx; L.M = M; L.K = K; L.dtype = dtype; L.y_dtype = y_dtype; L.nested = nested;
    L.mode = kTmaIndependent; L.nseg = 1;
    L.seg[0] = tma_segment(packed, ld_packed, absmax, ld_absmax, code2, absmax2, offset, gblk_base, gblk_row_stride,
                           N, y, ldy);
    L.code_dev = code;
    L.err = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + kErrWordOffset);
    const int r = nf4_tma_gemm(L, s);
    if (r != kTmaNotApplicable) return r;
  }
  if (M > 8 && tc5_path_enabled()) {
    Nf4Tc5Launch L;
    std::memset(&L, 0, sizeof(L));
    L.x = x; L.ldx = ldx; L.M = M; L.K = K; L.dtype = dtype; L.y_dtype = y_dtype; L.nested = nested;
    L.nseg = 1;
    L.seg[0] = Nf4Tc5Segment{packed, ld_packed, absmax, ld_absmax, absmax2, offset, gblk_base, gblk_row_stride,
                             N, y, ldy};
    L.code_dev = code;
    L.code2 = code2;
    L.err = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + kErrWordOffset);
    const int r = nf4_tc5_gemm(L, s);
    if (r != kTc5NotApplicable) return r;
  }
  GemmArgs a{};
  a.x = x; a.ldx = ldx;
  a.w = Nf4View{packed, ld_packed, absmax, ld_absmax, code2, absmax2, offset, gblk_base, gblk_row_stride, code};
  a.y = y; a.ldy = ldy;
  a.M = M; a.N = N; a.K = K;
  a.upg = K / (64 * c.cb);
  a.groups = static_cast<int>(c.groups);
  a.total = static_cast<int>(c.total);
  a.counters = static_cast<int*>(workspace);
  a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + c.counter_bytes);
  a.nseg = 1;
  a.pair = 0;
  a.static_w = 0;
  a.seg_end[0] = a.groups;
  a.seg[0] = SegView{a.w, y, ldy};
  if (dtype == B2D_F16)
    return y_dtype == B2D_F32 ? dispatch_tc<__half, float>(a, c, nested, s) : dispatch_tc<__half, __half>(a, c, nested, s);
  return y_dtype == B2D_F32 ? dispatch_tc<__nv_bfloat16, float>(a, c, nested, s)
                            : dispatch_tc<__nv_bfloat16, __nv_bfloat16>(a, c, nested, s);
}

namespace b2d {
namespace {
template <typename T, typename OT, bool NESTED>
int launch_simt(const GemmArgs& a, int grid, cudaStream_t s) {
  switch (a.M) {
    case 1: nf4_gemv_simt_kernel<T, OT, 1, NESTED><<<grid, kSimtThreads, 0, s>>>(a); break;
    case 2: nf4_gemv_simt_kernel<T, OT, 2, NESTED><<<grid, kSimtThreads, 0, s>>>(a); break;
    case 3: case 4: nf4_gemv_simt_kernel<T, OT, 4, NESTED><<<grid, kSimtThreads, 0, s>>>(a); break;
    default: nf4_gemv_simt_kernel<T, OT, 8, NESTED><<<grid, kSimtThreads, 0, s>>>(a); break;
  }
  return launch_status();
}

template <typename T, typename OT>
int launch_simt_n(const GemmArgs& a, int grid, int nested, cudaStream_t s) {
  return nested ? launch_simt<T, OT, true>(a, grid, s) : launch_simt<T, OT, false>(a, grid, s);
}
}  // namespace
}  // namespace b2d

extern "C" int b2d_nf4_gemv_simt(const void* x, int64_t ldx, const uint8_t* packed, int64_t ld_packed,
                                 const void* absmax, int64_t ld_absmax, int nested, const float* code2,
                                 const float* absmax2, float offset, int64_t gblk_base, int64_t gblk_row_stride,
                                 const float* code, void* y, int64_t ldy, int M, int N, int K, int dtype,
                                 int y_dtype, void* stream) {
  int st = check_weight_args(x, ldx, packed, ld_packed, absmax, ld_absmax, nested, code2, absmax2, code, y, ldy, M,
                             N, K, dtype, y_dtype, 8);
  if (st != B2D_OK || M == 0 || N == 0) return st;
  DeviceInfo di;
  if ((st = device_info(&di)) != B2D_OK) return st;
  GemmArgs a{};
  a.x = x; a.ldx = ldx;
  a.w = Nf4View{packed, ld_packed, absmax, ld_absmax, code2, absmax2, offset, gblk_base, gblk_row_stride, code};
  a.y = y; a.ldy = ldy;
  a.M = M; a.N = N; a.K = K;
  const int rows_per_cta = kSimtThreads / 32;
  int grid = (N + rows_per_cta - 1) / rows_per_cta;
  if (grid > di.sm_count * 8) grid = di.sm_count * 8;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B2D_F16)
    return y_dtype == B2D_F32 ? launch_simt_n<__half, float>(a, grid, nested, s)
                              : launch_simt_n<__half, __half>(a, grid, nested, s);
  return y_dtype == B2D_F32 ? launch_simt_n<__nv_bfloat16, float>(a, grid, nested, s)
                            : launch_simt_n<__nv_bfloat16, __nv_bfloat16>(a, grid, nested, s);
}

// ------------------------------------------------------------------------------------------ segmented
// Several weights on one x in one launch of the pipelined kernel (q/k/v or the paired gate/up of a
// decoder layer). No counterpart in the reference, which launches one kernel per projection.
extern "C" int b2d_nf4_gemm_multi(const void* x, int64_t ldx, const b2d_nf4_segment* segs, int nseg, int nested,
                                  int M, int K, int dtype, int y_dtype, int mode, int flags, const float* code_host,
                                  const void* epilogue, void* workspace, size_t workspace_bytes, void* stream) {
  if (!segs || nseg < 1 || nseg > kMaxSeg || M < 0 || K < 0) return B2D_ERR_ARG;
  if (mode != B2D_SEG_INDEPENDENT && mode != B2D_SEG_SILU_MUL && mode != B2D_SEG_ALLREDUCE) return B2D_ERR_ARG;
  const bool pair = mode == B2D_SEG_SILU_MUL;
  const bool ar = mode == B2D_SEG_ALLREDUCE;
  if (pair && (nseg != 2 || segs[0].N != segs[1].N || y_dtype != dtype)) return B2D_ERR_SHAPE;
  const b2d_allreduce_epilogue* are = static_cast<const b2d_allreduce_epilogue*>(epilogue);
  if (ar) {
    if (!are || !are->peer_bufs || !are->step || are->world < 1 || are->world > kArMaxWorld || are->rank < 0 ||
        are->rank >= are->world || are->sites < 1 || are->site < 0 || are->site >= are->sites || are->n_max % 8)
      return B2D_ERR_ARG;
    if (nseg != 1 || y_dtype != dtype) return B2D_ERR_SHAPE;
    if (static_cast<int64_t>((M + 1) / 2) * segs[0].N > are->n_max / 2) return B2D_ERR_SHAPE;
    for (int p = 0; p < are->world; ++p)
      if (!are->peer_bufs[p] || !aligned(are->peer_bufs[p], 256)) return B2D_ERR_ALIGN;
  }
  int64_t n_total = 0;
  for (int i = 0; i < nseg; ++i) {
    const b2d_nf4_segment& sg = segs[i];
    if (sg.N < 0) return B2D_ERR_ARG;
    if (sg.N % (pair ? 16 : 32) != 0) return B2D_ERR_SHAPE;
    // x, y, code and the shared constraints are checked per segment by the single-weight rules
    // outputs: a paired launch writes segment 0's y; an all-reduce launch writes the peers' buffers
    const void* yy = ar ? are->peer_bufs[are->rank] : (pair && i == 1 ? segs[0].y : sg.y);
    const int64_t ly = ar ? sg.N : (pair && i == 1 ? segs[0].ldy : sg.ldy);
    int st = check_weight_args(x, ldx, sg.packed, sg.ld_packed, sg.absmax, sg.ld_absmax, nested, sg.code2, sg.absmax2,
                               segs[0].code, yy, ly, M, sg.N, K, dtype, y_dtype, 8);
    if (st != B2D_OK) return st;
    if (!chunk4_ok(K, sg.absmax, sg.ld_absmax, nested, sg.gblk_base, sg.gblk_row_stride)) return B2D_ERR_ALIGN;
    n_total += sg.N;
  }
  if (M == 0 || n_total == 0) return B2D_OK;
  DeviceInfo di;
  int st;
  if ((st = device_info(&di)) != B2D_OK) return st;
  if (!workspace || workspace_bytes < kCounterBytes) return B2D_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return B2D_ERR_ALIGN;
  if (tma_path_enabled()) {
    Nf4TmaLaunch L;
    std::memset(&L, 0, sizeof(L));
    L.x = x; L.ldx = ldx; L.M = M; L.K = K; L.dtype = dtype; L.y_dtype = y_dtype; L.nested = nested;
    L.mode = pair ? kTmaSiluMul : (ar ? kTmaAllReduce : kTmaIndependent);
    L.nseg = nseg;
    for (int i = 0; i < nseg; ++i) {
      const b2d_nf4_segment& sg = segs[i];
      L.seg[i] = tma_segment(sg.packed, sg.ld_packed, sg.absmax, sg.ld_absmax, sg.code2, sg.absmax2, sg.offset,
                             sg.gblk_base, sg.gblk_row_stride, sg.N, pair ? segs[0].y : sg.y,
                             pair ? segs[0].ldy : sg.ldy);
    }
    L.code_dev = segs[0].code;
    L.code_host = code_host;
    L.pdl = (flags & B2D_LAUNCH_PDL) != 0;
    L.static_w = (flags & B2D_STATIC_WEIGHTS) != 0;
    if (ar) {
      for (int p = 0; p < are->world; ++p) L.ar.peer[p] = static_cast<uint8_t*>(are->peer_bufs[p]);
      L.ar.rank = are->rank;
      L.ar.world = are->world;
      L.ar.words = are->n_max / 2;
      L.ar.step = are->step;
      L.ar.site = are->site;
      L.ar.sites = are->sites;
    }
    L.err = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + kErrWordOffset);
    const int r = nf4_tma_gemm(L, static_cast<cudaStream_t>(stream));
    if (r != kTmaNotApplicable) return r;
  }
  GemmConfig c;
  if (n_total > (int64_t(1) << 30)) return B2D_ERR_SHAPE;
  if ((st = choose_config(M, static_cast<int>(n_total), K, true, di, &c)) != B2D_OK) return st;
  if (c.nt != 1 || c.rt != 2 || c.cb != 4) return B2D_ERR_SHAPE;
  if (!workspace || workspace_bytes < c.counter_bytes + c.partial_bytes) return B2D_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return B2D_ERR_ALIGN;
  GemmArgs a{};
  a.x = x; a.ldx = ldx;
  a.M = M; a.N = static_cast<int>(n_total); a.K = K;
  a.upg = K / 256;
  a.groups = static_cast<int>(c.groups);
  a.total = static_cast<int>(c.total);
  a.counters = static_cast<int*>(workspace);
  a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + c.counter_bytes);
  a.nseg = nseg;
  a.pair = pair ? 1 : 0;
  a.static_w = (flags & B2D_STATIC_WEIGHTS) ? 1 : 0;
  if (ar) {
    a.ar = 1;
    for (int p = 0; p < are->world; ++p) a.are.peer[p] = static_cast<uint8_t*>(are->peer_bufs[p]);
    a.are.rank = are->rank;
    a.are.world = are->world;
    a.are.words = are->n_max / 2;
    a.are.step = are->step;
    a.are.site = are->site;
    a.are.sites = are->sites;
  }
  if (code_host) {
    a.code_by_value = 1;
    for (int i = 0; i < 16; ++i) a.code_v[i] = code_host[i];
  }
  int end = 0;
  for (int i = 0; i < nseg; ++i) {
    const b2d_nf4_segment& sg = segs[i];
    a.seg[i] = SegView{Nf4View{sg.packed, sg.ld_packed, sg.absmax, sg.ld_absmax, sg.code2, sg.absmax2, sg.offset,
                               sg.gblk_base, sg.gblk_row_stride, segs[0].code},
                       sg.y, sg.ldy};
    end += pair ? sg.N / 16 : sg.N / 32;   // paired: both segments advance together
    a.seg_end[i] = pair ? sg.N / 16 : end;
  }
  a.w = a.seg[0].w;
  a.y = a.seg[0].y; a.ldy = a.seg[0].ldy;
  const bool pdl = (flags & B2D_LAUNCH_PDL) != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B2D_F16)
    return y_dtype == B2D_F32 ? dispatch_pipe<__half, float>(a, nested, pdl, s)
                              : dispatch_pipe<__half, __half>(a, nested, pdl, s);
  return y_dtype == B2D_F32 ? dispatch_pipe<__nv_bfloat16, float>(a, nested, pdl, s)
                            : dispatch_pipe<__nv_bfloat16, __nv_bfloat16>(a, nested, pdl, s);
}
