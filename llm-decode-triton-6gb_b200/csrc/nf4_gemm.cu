// Fused NF4 dequant + skinny matmul for sm_100a: y[M,N] = x[M,K] @ W[N,K]^T, W in bitsandbytes NF4.
//
// Replaces the reference's Triton kernel (profiling/kernels/nf4_gemm.py:37-64) and its launcher
// NF4Weight.matmul (nf4_gemm.py:94-106). Same storage semantics: row-major packed nibbles, even
// element in the high nibble, one scale per 64 weights, optional double-quant scale
// code2[q]*absmax2[blk/256]+offset (nf4_gemm.py:48-56); fp32 accumulation.
//
// Design (HBM-bound: ~0.52 B of weight state per weight, 2*M flops per weight):
//  * Persistent grid, one CTA per SM. The work is the list of (row group, 64-weight block) pairs in
//    row-group-major order; every CTA gets an equal contiguous slice and every warp an equal
//    contiguous sub-slice, so all SMs stream the same number of bytes for any (N, K). A row group
//    split between warps is summed in shared memory, one split between CTAs through a small global
//    workspace; the CTA that finishes a shared group last (atomic counter) adds the partials in
//    CTA order, so results are deterministic.
//  * Weights go global -> registers with 8-byte streaming loads (no shared-memory staging: the
//    shared-memory pipe is reserved for the dequant table), prefetched P pairs ahead.
//  * Dequant: a 256-entry table maps one packed byte to the pair (code[hi], code[lo]) in the
//    activation dtype, i.e. directly to one tensor-core A-fragment register. The table is
//    replicated once per lane (entry e, lane l at word 32e+l), so lookups never bank-conflict.
//  * The per-block scale is factored out of the dot product: the four m16n8k16 MMAs of one block
//    accumulate sum_k x_k*code[n_k] from zero, and the fp32 block scale multiplies that partial
//    into the running fp32 accumulator (one FMA per output element per block).
//  * The MMA reduction dimension is permuted so that each thread's 8 bytes of a block row are
//    contiguous in memory and the matching 16 activations are contiguous too:
//    thread (g, t) at k-step s owns bytes 8t+2s, 8t+2s+1 of its block row = k offsets 16t+4s+{0..3}.
#include "common.cuh"

namespace b2d {

namespace {

constexpr int kLutWords = 256 * 32;      // 256 byte values x 32 per-lane copies
constexpr int kGemmWarps = 8;
constexpr int kGemmThreads = kGemmWarps * 32;

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

struct GemmArgs {
  const void* x;
  int64_t ldx;
  Nf4View w;
  void* y;
  int64_t ldy;
  int M, N, K;
  int kb;            // K / 64
  int64_t groups;    // N / (16 * RT)
  int64_t total;     // groups * kb
  float* partials;   // [grid][2][E]
  int* counters;     // [groups]
};

template <int RT, int NT>
struct Stage {
  uint2 w[RT][2];        // rows g and g+8 of each 16-row tile: this thread's 8 bytes of the block
  uint32_t sraw[RT][2];  // fp32 bits of absmax, or the uint8 double-quant index
  float a2[RT][2];       // absmax2 of the block's group (double quant)
  uint4 xv[NT][2];       // 16 activations of token 8*nt+g for this thread's k offsets
};

template <typename T, int RT, int NT, bool NESTED>
__device__ __forceinline__ void load_stage(Stage<RT, NT>& st, const GemmArgs& a, int64_t grp, int blk,
                                           int g, int tq) {
  const T* x = static_cast<const T*>(a.x);
#pragma unroll
  for (int rt = 0; rt < RT; ++rt) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t row = grp * (16 * RT) + rt * 16 + h * 8 + g;
      st.w[rt][h] = ldg_stream_u2(a.w.packed + row * a.w.ld_packed + blk * 32 + tq * 8);
      const int64_t bi = row * a.w.ld_absmax + blk;
      if (NESTED) {
        st.sraw[rt][h] = __ldg(static_cast<const uint8_t*>(a.w.absmax) + bi);
        const int64_t gb = a.w.gblk_base + row * a.w.gblk_row_stride + blk;
        st.a2[rt][h] = __ldg(a.w.absmax2 + (gb >> 8));
      } else {
        st.sraw[rt][h] = __float_as_uint(__ldg(static_cast<const float*>(a.w.absmax) + bi));
      }
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int tok = nt * 8 + g;
    if (tok < a.M) {
      const T* p = x + tok * a.ldx + blk * 64 + tq * 16;
      st.xv[nt][0] = ldg_u4(p);
      st.xv[nt][1] = ldg_u4(p + 8);
    } else {
      st.xv[nt][0] = make_uint4(0, 0, 0, 0);
      st.xv[nt][1] = make_uint4(0, 0, 0, 0);
    }
  }
}

template <typename T, int RT, int NT, bool NESTED>
__device__ __forceinline__ void compute_stage(const Stage<RT, NT>& st, float (&acc)[RT][NT][4],
                                              const uint32_t* lutp, const float* code2_s, float offset) {
#pragma unroll
  for (int rt = 0; rt < RT; ++rt) {
    float c[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) c[nt][0] = c[nt][1] = c[nt][2] = c[nt][3] = 0.f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const uint32_t wg = (s < 2) ? st.w[rt][0].x : st.w[rt][0].y;
      const uint32_t wh = (s < 2) ? st.w[rt][1].x : st.w[rt][1].y;
      const int sh = (s & 1) * 2;
      const uint32_t a0 = lutp[byte_of(wg, sh) << 5];
      const uint32_t a2 = lutp[byte_of(wg, sh + 1) << 5];
      const uint32_t a1 = lutp[byte_of(wh, sh) << 5];
      const uint32_t a3 = lutp[byte_of(wh, sh + 1) << 5];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint32_t* xw = reinterpret_cast<const uint32_t*>(&st.xv[nt][0]);
        Mma<T>::run(c[nt], a0, a1, a2, a3, xw[2 * s], xw[2 * s + 1]);
      }
    }
    float sc[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (NESTED) {
        sc[h] = __fadd_rn(__fmul_rn(code2_s[st.sraw[rt][h]], st.a2[rt][h]), offset);
      } else {
        sc[h] = __uint_as_float(st.sraw[rt][h]);
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
}

// Store a finished 16*RT-row group held in fragment order (thread g,t owns rows g, g+8 of each
// tile and tokens 2t, 2t+1 of each n8 tile).
template <typename OT, int RT, int NT>
__device__ __forceinline__ void store_group(const GemmArgs& a, int64_t grp, const float (&v)[RT][NT][4],
                                            int g, int tq) {
  OT* y = static_cast<OT*>(a.y);
#pragma unroll
  for (int rt = 0; rt < RT; ++rt) {
    const int64_t r0 = grp * (16 * RT) + rt * 16 + g;
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

__device__ __forceinline__ int64_t cta_begin(int64_t c, int64_t total, int64_t grid) { return c * total / grid; }
// CTA whose slice contains pair p: the largest c with floor(c*total/grid) <= p.
__device__ __forceinline__ int64_t cta_of(int64_t p, int64_t total, int64_t grid) {
  return ((p + 1) * grid - 1) / total;
}

template <typename T, typename OT, int RT, int NT, bool NESTED, int P>
__global__ void __launch_bounds__(kGemmThreads, 1) nf4_gemm_tc_kernel(const GemmArgs a) {
  constexpr int E = RT * NT * 128;  // fp32 values of one group partial, in fragment order
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t* lut = reinterpret_cast<uint32_t*>(smem);
  float* code2_s = reinterpret_cast<float*>(smem + kLutWords * 4);
  float* slots = code2_s + 256;  // [warps][2][E]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;

  for (int i = tid; i < kLutWords; i += kGemmThreads) {
    const int e = i >> 5;
    lut[i] = Dt<T>::pack2(__ldg(a.w.code + (e >> 4)), __ldg(a.w.code + (e & 15)));
  }
  if (NESTED) {
    for (int i = tid; i < 256; i += kGemmThreads) code2_s[i] = __ldg(a.w.code2 + i);
  }
  __syncthreads();

  const int64_t grid = gridDim.x, cta = blockIdx.x;
  const int64_t A = cta_begin(cta, a.total, grid), B = cta_begin(cta + 1, a.total, grid);
  const int64_t wa = A + warp * (B - A) / kGemmWarps;
  const int64_t wb = A + (warp + 1) * (B - A) / kGemmWarps;
  const int kb = a.kb;
  const uint32_t* lutp = lut + lane;

  if (wa < wb) {
    Stage<RT, NT> st[P];
    // load cursor
    int64_t lgrp = wa / kb;
    int lblk = static_cast<int>(wa - lgrp * kb);
#pragma unroll
    for (int j = 0; j < P; ++j) {
      if (wa + j < wb) load_stage<T, RT, NT, NESTED>(st[j], a, lgrp, lblk, g, tq);
      if (++lblk == kb) { lblk = 0; ++lgrp; }
    }
    float acc[RT][NT][4];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) acc[rt][nt][0] = acc[rt][nt][1] = acc[rt][nt][2] = acc[rt][nt][3] = 0.f;

    const int64_t first_grp = wa / kb;
    int64_t cgrp = first_grp;
    int cblk = static_cast<int>(wa - cgrp * kb);

    auto flush = [&](int64_t grp) {
      const bool full = grp * kb >= wa && (grp + 1) * kb <= wb;
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
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[rt][nt][0] = acc[rt][nt][1] = acc[rt][nt][2] = acc[rt][nt][3] = 0.f;
    };

    for (int64_t base = wa; base < wb; base += P) {
#pragma unroll
      for (int j = 0; j < P; ++j) {
        if (base + j < wb) {
          compute_stage<T, RT, NT, NESTED>(st[j], acc, lutp, code2_s, a.w.offset);
          if (base + j + P < wb) load_stage<T, RT, NT, NESTED>(st[j], a, lgrp, lblk, g, tq);
          if (++lblk == kb) { lblk = 0; ++lgrp; }
          if (++cblk == kb) {
            flush(cgrp);
            cblk = 0;
            ++cgrp;
          }
        }
      }
    }
    if (cblk != 0) flush(cgrp);  // range ended inside a group
  }
  __syncthreads();

  // ---- combine the warp partials of this CTA (warp 0; lanes own their fragment positions)
  if (warp != 0 || A >= B) return;
  const int64_t gA = A / kb, gB = (B - 1) / kb;
  for (int64_t grp = gA; grp <= gB; ++grp) {
    float v[RT][NT][4];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) v[rt][nt][0] = v[rt][nt][1] = v[rt][nt][2] = v[rt][nt][3] = 0.f;
    bool done = false;
    for (int w = 0; w < kGemmWarps; ++w) {
      const int64_t xa = A + w * (B - A) / kGemmWarps, xb = A + (w + 1) * (B - A) / kGemmWarps;
      if (xa >= xb) continue;
      if (grp * kb >= xa && (grp + 1) * kb <= xb) { done = true; break; }
      const int64_t fg = xa / kb, lg = (xb - 1) / kb;
      if (grp < fg || grp > lg) continue;
      const float* s = slots + (w * 2 + (grp == fg ? 0 : 1)) * E + lane * 4;
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float4 q = *reinterpret_cast<const float4*>(s + (rt * NT + nt) * 128);
          v[rt][nt][0] += q.x; v[rt][nt][1] += q.y; v[rt][nt][2] += q.z; v[rt][nt][3] += q.w;
        }
    }
    if (done) continue;
    if (grp * kb >= A && (grp + 1) * kb <= B) {
      store_group<OT, RT, NT>(a, grp, v, g, tq);
      continue;
    }
    // group shared with neighbouring CTAs: publish this CTA's partial, last arriver reduces
    float* mine = a.partials + (cta * 2 + (grp == gA ? 0 : 1)) * E + lane * 4;
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        __stcg(reinterpret_cast<float4*>(mine + (rt * NT + nt) * 128),
               make_float4(v[rt][nt][0], v[rt][nt][1], v[rt][nt][2], v[rt][nt][3]));
    __threadfence();
    __syncwarp();
    const int64_t c_lo = cta_of(grp * kb, a.total, grid), c_hi = cta_of((grp + 1) * kb - 1, a.total, grid);
    int last = 0;
    if (lane == 0) {
      const int old = atomicAdd(a.counters + grp, 1);
      if (old == static_cast<int>(c_hi - c_lo)) {
        last = 1;
        a.counters[grp] = 0;
      }
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) continue;
    __threadfence();
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) v[rt][nt][0] = v[rt][nt][1] = v[rt][nt][2] = v[rt][nt][3] = 0.f;
    for (int64_t c = c_lo; c <= c_hi; ++c) {
      const int64_t cfirst = cta_begin(c, a.total, grid) / kb;
      const float* s = a.partials + (c * 2 + (grp == cfirst ? 0 : 1)) * E + lane * 4;
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float4 q = __ldcg(reinterpret_cast<const float4*>(s + (rt * NT + nt) * 128));
          v[rt][nt][0] += q.x; v[rt][nt][1] += q.y; v[rt][nt][2] += q.z; v[rt][nt][3] += q.w;
        }
    }
    store_group<OT, RT, NT>(a, grp, v, g, tq);
  }
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
constexpr int64_t kMaxGroups = kCounterBytes / 4;

struct GemmConfig {
  int rt, nt;
  int64_t groups, total;
  int grid;
  size_t counter_bytes, partial_bytes;
};

int choose_config(int M, int N, int K, const DeviceInfo& di, GemmConfig* c) {
  c->nt = M <= 8 ? 1 : (M <= 16 ? 2 : (M <= 32 ? 4 : 8));
  c->rt = (c->nt == 1 && N % 32 == 0) ? 2 : 1;
  c->groups = N / (16 * c->rt);
  c->total = c->groups * (K / 64);
  int64_t grid = di.sm_count;
  if (grid > c->total) grid = c->total;
  if (grid < 1) grid = 1;
  c->grid = static_cast<int>(grid);
  c->counter_bytes = kCounterBytes;
  c->partial_bytes = static_cast<size_t>(c->grid) * 2 * (c->rt * c->nt * 128) * 4;
  return c->groups <= kMaxGroups ? B2D_OK : B2D_ERR_SHAPE;
}

size_t gemm_smem_bytes(int rt, int nt) {
  return kLutWords * 4 + 256 * 4 + static_cast<size_t>(kGemmWarps) * 2 * rt * nt * 128 * 4;
}

template <typename T, typename OT, int RT, int NT, bool NESTED, int P>
int launch_tc(const GemmArgs& a, int grid, cudaStream_t stream) {
  auto kern = nf4_gemm_tc_kernel<T, OT, RT, NT, NESTED, P>;
  const size_t smem = gemm_smem_bytes(RT, NT);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) { set_cuda_error(e); return B2D_ERR_LAUNCH; }
  kern<<<grid, kGemmThreads, smem, stream>>>(a);
  return launch_status();
}

template <typename T, typename OT, bool NESTED>
int dispatch_tc(const GemmArgs& a, const GemmConfig& c, cudaStream_t s) {
  if (c.nt == 1)
    return c.rt == 2 ? launch_tc<T, OT, 2, 1, NESTED, 4>(a, c.grid, s) : launch_tc<T, OT, 1, 1, NESTED, 6>(a, c.grid, s);
  if (c.nt == 2) return launch_tc<T, OT, 1, 2, NESTED, 4>(a, c.grid, s);
  if (c.nt == 4) return launch_tc<T, OT, 1, 4, NESTED, 2>(a, c.grid, s);
  return launch_tc<T, OT, 1, 8, NESTED, 2>(a, c.grid, s);
}

template <typename T, typename OT>
int dispatch_tc_n(const GemmArgs& a, const GemmConfig& c, int nested, cudaStream_t s) {
  return nested ? dispatch_tc<T, OT, true>(a, c, s) : dispatch_tc<T, OT, false>(a, c, s);
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
  if (choose_config(M, N, K, di, &c) != B2D_OK) return 0;
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
  if ((st = choose_config(M, N, K, di, &c)) != B2D_OK) return st;
  if (!workspace || workspace_bytes < c.counter_bytes + c.partial_bytes) return B2D_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return B2D_ERR_ALIGN;
  GemmArgs a;
  a.x = x; a.ldx = ldx;
  a.w = Nf4View{packed, ld_packed, absmax, ld_absmax, code2, absmax2, offset, gblk_base, gblk_row_stride, code};
  a.y = y; a.ldy = ldy;
  a.M = M; a.N = N; a.K = K;
  a.kb = K / 64;
  a.groups = c.groups;
  a.total = c.total;
  a.counters = static_cast<int*>(workspace);
  a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + c.counter_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B2D_F16)
    return y_dtype == B2D_F32 ? dispatch_tc_n<__half, float>(a, c, nested, s) : dispatch_tc_n<__half, __half>(a, c, nested, s);
  return y_dtype == B2D_F32 ? dispatch_tc_n<__nv_bfloat16, float>(a, c, nested, s)
                            : dispatch_tc_n<__nv_bfloat16, __nv_bfloat16>(a, c, nested, s);
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
