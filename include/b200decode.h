/*
 * b200decode.h -- C ABI of the B200 (sm_100a) decode kernels: the fused NF4 dequant +
 * skinny matmul and the split-K flash-decoding GQA attention (partial + log-sum-exp combine).
 *
 * Plain C: raw device pointers, sizes, strides in elements, an int status. The library never
 * allocates device memory: the caller owns every input, output and workspace, and passes the
 * CUDA stream (a cudaStream_t, written here as void*; NULL is the legacy default stream) that
 * the work is enqueued on. All calls are asynchronous with respect to the host; a nonzero
 * status means nothing was launched (argument checks) or the launch itself failed.
 *
 * Reference interfaces replaced (paths inside Muhammad-Hamza-cpp/llm-decode-triton-6gb):
 *   b2d_nf4_gemm            <- NF4Weight.matmul + _nf4_gemm_kernel   profiling/kernels/nf4_gemm.py:94-106, :37-64
 *   b2d_nf4_dequant         <- bitsandbytes.functional.dequantize_4bit, the stock dequant the
 *                              reference validates against            profiling/kernels/bench_nf4.py:34
 *   b2d_gqa_decode_partial  <- _partial_kernel                       profiling/kernels/decode_attention.py:18-55
 *   b2d_gqa_decode_combine  <- _merge_kernel                         profiling/kernels/decode_attention.py:58-72
 *   b2d_gqa_decode          <- decode_attention (wrapper)            profiling/kernels/decode_attention.py:75-91
 *   b2d_nf4_quantize,
 *   b2d_nf4_double_quant    <- the bitsandbytes quantiser that produced the checkpoint the
 *                              reference loads (Params4bit / quantize_4bit, profiling/common.py:37-42);
 *                              used to build models on the device
 */
#ifndef B200DECODE_H_
#define B200DECODE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status codes */
enum {
  B2D_OK = 0,
  B2D_ERR_ARG = 1,        /* null pointer where one is required, negative size */
  B2D_ERR_SHAPE = 2,      /* unsupported shape (e.g. N % 16, K % 64, head_dim, group size) */
  B2D_ERR_DTYPE = 3,      /* dtype code not supported by this entry point */
  B2D_ERR_ALIGN = 4,      /* pointer or leading dimension breaks the vector-load alignment */
  B2D_ERR_WORKSPACE = 5,  /* workspace missing or smaller than the *_workspace_bytes query */
  B2D_ERR_LAUNCH = 6,     /* the CUDA launch reported an error (message: b2d_last_cuda_error) */
  B2D_ERR_DEVICE = 7      /* no CUDA device, or not a compute capability 10.x device */
};

/* dtype codes for activations / outputs */
enum { B2D_F16 = 0, B2D_BF16 = 1, B2D_F32 = 2 };

/* Launch flags of the decode-step entry points (the *_ex / multi / glue calls):
 *   B2D_LAUNCH_PDL      launch as a programmatic dependent of the previous kernel in the stream:
 *                       the kernel may be scheduled while that kernel drains and waits (on the
 *                       device) for its completion before touching stream-ordered data. Safe after
 *                       any kernel; it only gains when the previous kernel is one of this library's.
 *   B2D_STATIC_WEIGHTS  (NF4 GEMM) the weights are not written by the preceding kernels of the
 *                       stream, so their prefetch may start before the previous kernel completes.
 *   B2D_ATTN_FUSED_COMBINE  (attention) one launch: the last split CTA of each (sequence, KV head)
 *                       to finish does the log-sum-exp combine (no second kernel). Applies when
 *                       nsplit <= 64 and B*KVH <= 16384; otherwise the two-kernel path runs.
 *   B2D_KV_STATIC_PREFIX  (attention, with B2D_LAUNCH_PDL) the preceding kernels of the stream write
 *                       at most the last cached key/value of each sequence (a decode step's append),
 *                       so the keys before it may be prefetched before the previous kernel completes. */
enum { B2D_LAUNCH_PDL = 1, B2D_STATIC_WEIGHTS = 2, B2D_ATTN_FUSED_COMBINE = 4, B2D_KV_STATIC_PREFIX = 8 };

const char* b2d_strerror(int status);
/* Text of the last CUDA error seen by a launch in this thread ("" if none). */
const char* b2d_last_cuda_error(void);
/* ABI version: (major << 16) | minor. */
int b2d_version(void);

/* ================================================================ NF4 storage format
 * A weight W[N,K] in bitsandbytes NF4: flattened row-major, 64 weights per block, two 4-bit
 * codes per byte with the EVEN element in the HIGH nibble (nf4_gemm.py:4,55-56).
 *   packed     uint8, row r starts at packed + r*ld_packed (bytes); ld_packed >= K/2
 *   absmax     per-block scale: fp32 if nested == 0, uint8 index into code2 if nested != 0;
 *              row r's blocks start at absmax + r*ld_absmax (elements)
 *   code2, absmax2, offset   double quantisation (nested != 0):
 *              scale = fp32(fp32(code2[q] * absmax2[gblk / 256]) + offset)  (nf4_gemm.py:50-51)
 *              where gblk = gblk_base + r*gblk_row_stride + k/64 is the block's index in the
 *              FULL tensor (so a tensor-parallel shard indexes absmax2 exactly as the whole)
 *   code       16 fp32 codebook values (quant_state.code)
 * Unsharded tensor: ld_packed = K/2, ld_absmax = gblk_row_stride = K/64, gblk_base = 0.
 * ================================================================================== */

/* out[r, k] = round_dtype(fp32(code[nib] * scale)) for r < n_rows, k < k_cols.
 * Bit-exact with bitsandbytes.functional.dequantize_4bit. out is row-major with ld_out. */
int b2d_nf4_dequant(const uint8_t* packed, int64_t ld_packed,
                    const void* absmax, int64_t ld_absmax, int nested,
                    const float* code2, const float* absmax2, float offset,
                    int64_t gblk_base, int64_t gblk_row_stride, const float* code,
                    void* out, int64_t ld_out, int64_t n_rows, int64_t k_cols, int dtype,
                    void* stream);

/* Scratch bytes b2d_nf4_gemm needs for (M, N, K) on the current device. Zero-fill a new
 * workspace once; every launch leaves its counters at zero again, so one workspace can serve
 * any sequence of calls on one stream (calls that may overlap need separate workspaces). */
size_t b2d_nf4_gemm_workspace_bytes(int M, int N, int K);

/* y[m, n] = sum_k x[m, k] * W[n, k] for m < M, fp32 accumulation.
 * x: [M, K] row-major with ldx (elements, multiple of 8, 16-byte aligned base), dtype F16/BF16.
 * y: [M, N] row-major with ldy, y_dtype = dtype or F32.
 * Constraints: 1 <= M <= 64, N % 16 == 0, K % 64 == 0 (the reference needs N%64, K%256).
 * Tensor-core path (mma.sync m16n8k16, fp32 accumulate) over a dequant look-up table. */
int b2d_nf4_gemm(const void* x, int64_t ldx,
                 const uint8_t* packed, int64_t ld_packed,
                 const void* absmax, int64_t ld_absmax, int nested,
                 const float* code2, const float* absmax2, float offset,
                 int64_t gblk_base, int64_t gblk_row_stride, const float* code,
                 void* y, int64_t ldy, int M, int N, int K, int dtype, int y_dtype,
                 void* workspace, size_t workspace_bytes, void* stream);

/* One weight of a segmented NF4 GEMM: the b2d_nf4_gemm weight arguments plus its row count and
 * output. */
typedef struct {
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
  int N;
  void* y;
  int64_t ldy;
} b2d_nf4_segment;

enum { B2D_SEG_INDEPENDENT = 0, B2D_SEG_SILU_MUL = 1, B2D_SEG_ALLREDUCE = 2 };

/* Where a tensor-parallel all-reduce fused into a GEMM epilogue sends its partial sums (no counterpart
 * in the reference, which is single-GPU). Buffers as for b2d_allreduce (one per rank, sized by
 * b2d_allreduce_buffer_bytes(n_max, world, dtype), zero-filled once, mapped by every peer; a separate
 * buffer from the one b2d_allreduce uses). The call's epoch is read on the device:
 * step[0] * sites + site + 1, so a captured CUDA graph stays valid while the caller advances
 * *step once per decode step (every rank the same way) and gives each all-reduce of a step its own
 * site in [0, sites). Epochs must keep increasing over the buffer's life. */
typedef struct {
  void* const* peer_bufs;   /* HOST array [world]: every rank's buffer as seen from this GPU */
  int rank, world;          /* world <= 8 */
  int64_t n_max;            /* elements the buffers were sized for (multiple of 8) */
  const int64_t* step;      /* device counter */
  int site, sites;
} b2d_allreduce_epilogue;

/* Several NF4 weights applied to the same x in ONE launch (no counterpart in the reference, which
 * launches one kernel per projection; this fuses q/k/v and gate/up of a decoder layer).
 *   mode B2D_SEG_INDEPENDENT: segs[i].y = x @ W_i^T for every segment (1 <= nseg <= 4, N_i % 32 == 0).
 *   mode B2D_SEG_SILU_MUL:    nseg == 2, N_0 == N_1 (multiple of 16), y_dtype == dtype:
 *                             segs[0].y = silu(x @ W_0^T) * (x @ W_1^T), every intermediate rounded to
 *                             dtype as in a Mistral MLP (act_fn(gate_proj(x)) * up_proj(x)).
 * 1 <= M <= 8. All segments share `nested` and segs[0].code (the 16-value NF4 codebook); per-segment
 * scales (absmax/code2/absmax2/offset) are their own. Every segment's scales must allow 4-block
 * loads: (K/64) % 4 == 0 and ld_absmax % 4 == 0; nested: gblk_base % 4 == 0 and gblk_row_stride % 4 == 0,
 * plain: 16-byte aligned absmax. Workspace: b2d_nf4_gemm_workspace_bytes(M, sum of N_i, K).
 *   mode B2D_SEG_ALLREDUCE:   nseg == 1, y_dtype == dtype, epilogue = a b2d_allreduce_epilogue: the
 *                             partial product x @ W_0^T (this rank's K slice of a row-parallel
 *                             linear, rounded to dtype) is not stored to segs[0].y but written into
 *                             every peer's buffer, to be summed by b2d_allreduce_add_rmsnorm with the
 *                             same epilogue descriptor. (M + 1) / 2 * N_0 <= n_max / 2.
 * flags: B2D_LAUNCH_PDL | B2D_STATIC_WEIGHTS. code_host: NULL, or a HOST copy of the 16 values of
 * segs[0].code, passed with the launch so the dequant table is built without a device read.
 * epilogue: NULL unless mode is B2D_SEG_ALLREDUCE. */
int b2d_nf4_gemm_multi(const void* x, int64_t ldx, const b2d_nf4_segment* segs, int nseg, int nested,
                       int M, int K, int dtype, int y_dtype, int mode, int flags, const float* code_host,
                       const void* epilogue, void* workspace, size_t workspace_bytes, void* stream);

/* CUDA-core variant (fp32 FMAs, warp-shuffle reductions, no tensor cores) of b2d_nf4_gemm for
 * 1 <= M <= 8: same arguments and constraints, no workspace. Kept as the measured comparison
 * point for the tensor-core path. */
int b2d_nf4_gemv_simt(const void* x, int64_t ldx,
                      const uint8_t* packed, int64_t ld_packed,
                      const void* absmax, int64_t ld_absmax, int nested,
                      const float* code2, const float* absmax2, float offset,
                      int64_t gblk_base, int64_t gblk_row_stride, const float* code,
                      void* y, int64_t ldy, int M, int N, int K, int dtype, int y_dtype,
                      void* stream);

/* Blockwise NF4 quantisation of n (multiple of 64) contiguous values of dtype F32/F16/BF16:
 * absmax[b] = max |w| over block b; code index = nearest code to fp32(w * fp32(1/absmax)),
 * ties to the lower code; packed[i] = idx[2i] << 4 | idx[2i+1]. */
int b2d_nf4_quantize(const void* w, int64_t n, int dtype, const float* code,
                     uint8_t* packed, float* absmax, void* stream);

/* Double quantisation of n_blocks fp32 scales: offset = fixed-order float64 mean, rounded to
 * fp32 (written to *offset_out, a device float); per group of 256: absmax2 = max |a - offset|,
 * q = nearest code2 entry to fp32((a - offset) * fp32(1/absmax2)). code2 is ascending. */
int b2d_nf4_double_quant(const float* absmax, int64_t n_blocks, const float* code2,
                         uint8_t* qabsmax, float* absmax2, float* offset_out, void* stream);

/* ================================================================ GQA decode attention
 * One query token per sequence. q: [B, H, 1, D] (strides sq_b, sq_h), k/v: [B, KVH, S, D]
 * (strides s*_b, s*_h, s*_s), out: [B, 1, H, D] (strides so_b, so_h). Last dim contiguous,
 * strides in elements. Query head h reads KV head h / (H / KVH). seqlens: int32 [B] valid
 * keys per sequence (NULL = all S). Keys [split*chunk, (split+1)*chunk) form one split.
 * D in {64, 128}; G = H / KVH in 1..16; dtype F16 or BF16 for q, k, v; out_dtype = dtype or F32.
 * Workspace: a 64 KiB region of int32 arrival counters (used by the single-launch combine), then
 * fp32 acc [B, H, nsplit, D] and ml [B, H, nsplit, 2]. Zero-fill a new workspace once; launches leave
 * the counters at zero, so one workspace serves any sequence of calls on one stream.
 * ================================================================================== */

/* Split count the library picks for (B, KVH, S) on the current device (chunk = ceil(S/nsplit)
 * rounded up to a multiple of 32 keys). */
int b2d_gqa_default_splits(int B, int KVH, int S);
size_t b2d_gqa_workspace_bytes(int B, int H, int nsplit, int D);

int b2d_gqa_decode_partial(const void* q, int64_t sq_b, int64_t sq_h,
                           const void* k, int64_t sk_b, int64_t sk_h, int64_t sk_s,
                           const void* v, int64_t sv_b, int64_t sv_h, int64_t sv_s,
                           const int32_t* seqlens, int B, int H, int KVH, int S, int D,
                           float scale, int nsplit, int chunk, int dtype,
                           void* workspace, size_t workspace_bytes, void* stream);

int b2d_gqa_decode_combine(const int32_t* seqlens, int B, int H, int S, int D,
                           int nsplit, int chunk, int out_dtype,
                           const void* workspace, size_t workspace_bytes,
                           void* out, int64_t so_b, int64_t so_h, void* stream);

/* partial + combine in one call (the combine is launched with programmatic dependent launch so
 * its launch overlaps the partial kernel's tail). nsplit <= 0 or chunk <= 0 picks defaults. */
int b2d_gqa_decode(const void* q, int64_t sq_b, int64_t sq_h,
                   const void* k, int64_t sk_b, int64_t sk_h, int64_t sk_s,
                   const void* v, int64_t sv_b, int64_t sv_h, int64_t sv_s,
                   const int32_t* seqlens, int B, int H, int KVH, int S, int D,
                   float scale, int nsplit, int chunk, int dtype,
                   void* workspace, size_t workspace_bytes,
                   void* out, int64_t so_b, int64_t so_h, int out_dtype, void* stream);

/* b2d_gqa_decode with launch flags (B2D_LAUNCH_PDL: the partial kernel is launched as a programmatic
 * dependent of the previous kernel in the stream). */
int b2d_gqa_decode_ex(const void* q, int64_t sq_b, int64_t sq_h,
                      const void* k, int64_t sk_b, int64_t sk_h, int64_t sk_s,
                      const void* v, int64_t sv_b, int64_t sv_h, int64_t sv_s,
                      const int32_t* seqlens, int B, int H, int KVH, int S, int D,
                      float scale, int nsplit, int chunk, int dtype,
                      void* workspace, size_t workspace_bytes,
                      void* out, int64_t so_b, int64_t so_h, int out_dtype, int flags, void* stream);

/* Decode-step attention with the step's RoPE and KV-cache append folded into the partial kernel (no
 * counterpart in the reference, whose decode step rotates q/k and appends to the cache with torch ops
 * before its attention kernel). q [B, H*D] (row stride ldq) and k_new / v_new [B, KVH*D] are this step's
 * projection outputs before RoPE; pos [B] (int64) the step's position of each sequence, written before
 * the step; rcos / rsin [>= S, D] (row stride ld_cs) the rotary tables. The launch rotates q in
 * registers, writes the rotated key and the value at position pos[b] of k_cache / v_cache (the HF
 * layout [B, KVH, S, D] with the given strides), writes seqlens[b] = pos[b] + 1 (0 for a position
 * outside [0, S)) and attends over keys [0, pos[b]]; the keys before pos[b] are fetched before the
 * previous kernel completes under B2D_LAUNCH_PDL, so the preceding kernels must not write them. Same
 * rounding as b2d_rope_kv_append followed by b2d_gqa_decode_ex: the outputs and the caches are
 * bit-identical. Default split choice; workspace as b2d_gqa_decode. flags: B2D_LAUNCH_PDL. */
int b2d_gqa_decode_append(const void* q, int64_t ldq, const void* k_new, int64_t ldk,
                          const void* v_new, int64_t ldv, const int64_t* pos,
                          const void* rcos, const void* rsin, int64_t ld_cs,
                          void* k_cache, int64_t sk_b, int64_t sk_h, int64_t sk_s,
                          void* v_cache, int64_t sv_b, int64_t sv_h, int64_t sv_s,
                          int32_t* seqlens, int B, int H, int KVH, int S, int D, float scale, int dtype,
                          void* workspace, size_t workspace_bytes,
                          void* out, int64_t so_b, int64_t so_h, int out_dtype, int flags, void* stream);

/* One-shot L2 prefetch hint (no counterpart in the reference): the next b2d_gqa_decode_append call made by
 * this host thread also prefetches up to 4 device ranges into L2 (ptrs 16-byte aligned; the whole 16-byte
 * units of each range), spread over its CTAs and issued before any dependency wait, then the hint is
 * cleared. Meant for static data the launches after it read (the next GEMMs' weights); no result
 * depends on it. */
int b2d_l2_prefetch_hint(const void* const* ptrs, const int64_t* bytes, int n);

/* ================================================================ decode-step glue
 * The small per-layer operations of a Mistral decoder layer around the two hot paths, as kernels
 * that take B2D_LAUNCH_PDL (no counterpart in the reference, which runs these as separate torch ops:
 * transformers' MistralRMSNorm, apply_rotary_pos_emb, DynamicCache.update, SiLU and the residual
 * adds). dtype F16 or BF16; every intermediate is rounded to dtype where the torch code rounds.
 * ================================================================================== */

/* Residual add + RMSNorm over rows of width D (M rows, D % 8 == 0, D <= 8192):
 *   h = residual + x (rounded; x may be NULL: h = residual), written back into residual;
 *   out = round(weight * round(h * rsqrt(mean(h^2) + eps)))   (MistralRMSNorm, fp32 statistics).
 * With B2D_LAUNCH_PDL the norm weight is read before the previous kernel completes: it must not be
 * written by that kernel. */
int b2d_add_rmsnorm(const void* x, int64_t ldx, void* residual, int64_t ldr, const void* weight, float eps,
                    void* out, int64_t ldo, int M, int D, int dtype, int flags, void* stream);

/* Rotary embedding of one new token per sequence plus the KV-cache append.
 * q: [B, H*D] (row stride ldq), k, v: [B, KVH*D] (ldk, ldv), the projection outputs;
 * pos: int64 [B], the token's position; cos, sin: [S_max, D] tables (row stride ld_cs) holding the
 * model's rotary values in dtype (HF rotary_emb output for positions 0..S_max-1).
 *   q_out[b, h, :]             = q*cos + rotate_half(q)*sin  (strides sqo_b, sqo_h; may alias q)
 *   k_cache[b, kvh, pos[b], :] = k*cos + rotate_half(k)*sin  (strides skc_b, skc_h, skc_s)
 *   v_cache[b, kvh, pos[b], :] = v                            (strides svc_b, svc_h, svc_s)
 *   seqlens[b] = pos[b] + 1 (int32; seqlens may be NULL).
 * A position outside [0, S_max) writes nothing for that sequence and sets seqlens[b] = 0.
 * D % 4 == 0, D <= 256, H % KVH == 0. */
int b2d_rope_kv_append(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                       const int64_t* pos, const void* cos, const void* sin, int64_t ld_cs,
                       void* q_out, int64_t sqo_b, int64_t sqo_h,
                       void* k_cache, int64_t skc_b, int64_t skc_h, int64_t skc_s,
                       void* v_cache, int64_t svc_b, int64_t svc_h, int64_t svc_s,
                       int32_t* seqlens, int B, int H, int KVH, int D, int S_max, int dtype, int flags,
                       void* stream);

/* out[m, n] = round(round(silu(gate[m, n])) * up[m, n]) for M rows of N (N % 8 == 0). */
int b2d_silu_mul(const void* gate, int64_t ldg, const void* up, int64_t ldu, void* out, int64_t ldo,
                 int M, int N, int dtype, int flags, void* stream);

/* ================================================================ lm_head + greedy argmax
 * logits[m, v] = x[m, :] . W[v, :] (fp32 accumulation, rounded to dtype) and ids[m] = the index of the
 * largest logit of row m, ties to the lowest index -- replaces the reference decode step's
 * `lm_head` GEMV followed by `logits.argmax(-1)` (profiling/common.py decode_step; the stock
 * LlamaForCausalLM/MistralForCausalLM head) with one launch. W is the [V, K] row-major head weight
 * (row stride ldw), x [M, K]; 1 <= M <= 64, K % 256 == 0, 16-byte aligned x and W, ldx/ldw % 8 == 0.
 * Outputs (any may be NULL, not all): logits [M, V] (row stride ld_logits), ids int64 [M], keys [M] =
 * the packed (value, index) maxima, ordered as signed 64-bit integers -- for a vocabulary-parallel
 * shard, indices are offset by vocab_offset and the shards' results merge by taking the maximum key
 * over ranks (id = 0xFFFFFFFF - (key & 0xFFFFFFFF)). Workspace: b2d_lm_head_workspace_bytes(V) bytes,
 * 256-byte aligned, zero-filled once before first use (it returns to zero after every call); calls
 * sharing a workspace must not overlap. flags: B2D_LAUNCH_PDL | B2D_STATIC_WEIGHTS. */
size_t b2d_lm_head_workspace_bytes(int V);
int b2d_lm_head_argmax(const void* x, int64_t ldx, const void* w, int64_t ldw, int M, int V, int K,
                       int64_t vocab_offset, void* logits, int64_t ld_logits, int64_t* ids, long long* keys,
                       int dtype, int flags, void* workspace, size_t workspace_bytes, void* stream);

/* ================================================================ tensor-parallel all-reduce
 * One-shot sum of n elements across `world` GPUs over NVLink peer memory (no counterpart in the
 * reference, which is single-GPU; used in place of the NCCL all-reduce after o_proj and down_proj).
 * Every rank owns a buffer of b2d_allreduce_buffer_bytes(n_max, world, dtype) bytes, zero-filled once
 * before first use and mapped by all peers; peer_bufs is a HOST array of the world buffers' device
 * addresses as seen from this GPU (peer_bufs[rank] = this rank's own). All ranks must make the same
 * sequence of calls (same n). out = sum over ranks of in, in rank order in fp32, rounded once: every
 * rank gets identical bits. in may equal out. n % 8 == 0, n <= n_max, n <= 64 * 4096; dtype F16 or
 * BF16; world <= 8. A wait that times out (a peer that never arrives) counts one error in the int32
 * at byte offset 256 of this rank's buffer and the kernel returns (its output is then invalid).
 * flags: B2D_LAUNCH_PDL. */
size_t b2d_allreduce_buffer_bytes(int64_t n_max, int world, int dtype);
int b2d_allreduce(const void* in, void* out, int64_t n, int dtype, void* const* peer_bufs, int rank,
                  int world, int64_t n_max, int flags, void* stream);

/* The consumer half of an all-reduce fused into a GEMM epilogue (B2D_SEG_ALLREDUCE), merged with the
 * residual add + RMSNorm that follows o_proj / down_proj:
 *   x = sum over ranks (rank order, fp32, one rounding) of the partials of the epilogue's site;
 *   residual += x; out = rmsnorm(residual) * weight   -- exactly b2d_allreduce then b2d_add_rmsnorm.
 * M rows of D (= the GEMM's N; D % 8 == 0, D <= 8192, (M + 1) / 2 * D <= n_max / 2). Waits are
 * bounded: a peer that never writes counts one error in the int32 at byte offset 256 of this rank's
 * buffer and the kernel returns. flags: B2D_LAUNCH_PDL. */
int b2d_allreduce_add_rmsnorm(const b2d_allreduce_epilogue* ar, void* residual, int64_t ldr, const void* weight,
                              float eps, void* out, int64_t ldo, int M, int D, int dtype, int flags, void* stream);

/* b2d_gqa_decode without a caller workspace (no counterpart in the reference). For callers that
 * cannot allocate device memory themselves -- a serving process whose allocator owns the whole device
 * budget, or a plugin inside another framework's memory pool that must not cudaMalloc behind its
 * back -- the split partials go to a static 8 MiB device array in the library (held by every GPU
 * that loads it until exit). The function allocates nothing. Needs 64 KiB + B*H*nsplit*(D+2)*4 bytes
 * <= 8 MiB, else returns B2D_ERR_WORKSPACE with the sizes in b2d_last_cuda_error(). The first call on a device
 * looks the array's address up once (make it before any stream capture). All calls on a device share
 * the array: calls that overlap on the GPU race. Other arguments as b2d_gqa_decode. */
int b2d_gqa_decode_noalloc(const void* q, int64_t sq_b, int64_t sq_h,
                           const void* k, int64_t sk_b, int64_t sk_h, int64_t sk_s,
                           const void* v, int64_t sv_b, int64_t sv_h, int64_t sv_s,
                           const int32_t* seqlens, int B, int H, int KVH, int S, int D,
                           float scale, int nsplit, int chunk, int dtype,
                           void* out, int64_t so_b, int64_t so_h, int out_dtype, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* B200DECODE_H_ */
