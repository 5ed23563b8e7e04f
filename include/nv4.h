/*
 * nv4 -- C ABI of the B200 (sm_100a) quantized-linear kernels of
 * nano-vllm-int4: W4A4 activation prep (randomized Hadamard transform +
 * per-128-group INT4 quantisation + packing), the grouped INT4 x INT4 GEMM with
 * BF16 group scales, and the GPTQ W4A16 dequant GEMM.
 *
 * Conventions for every entry point:
 *   - plain device pointers and sizes; no framework types;
 *   - all buffers are caller-owned; nothing is retained across calls (the
 *     set-up calls nv4_peer_buffer_alloc / _free / _open / _close manage the
 *     tensor-parallel peer buffers and are the only ones that allocate);
 *   - work is enqueued on `stream` (a cudaStream_t passed as void*; NULL is the
 *     legacy default stream) with no host synchronisation, no allocation and no
 *     device-wide synchronisation, so every entry point may be captured in a
 *     CUDA graph (the layer that calls them captures them at batch sizes 1..32);
 *   - the return value is NV4_OK or a negative NV4_ERR_* code; nothing is
 *     launched when an argument check fails.
 * Tensors are dense row-major; "bf16" buffers hold IEEE bfloat16 bit patterns.
 */
#ifndef NV4_H_
#define NV4_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NV4_OK 0
#define NV4_ERR_INVALID_ARGUMENT (-1) /* shape, null pointer or flag out of range */
#define NV4_ERR_UNSUPPORTED (-2)      /* valid request this build does not handle */
#define NV4_ERR_ALIGNMENT (-3)        /* a pointer is not aligned as documented */
#define NV4_ERR_CUDA (-4)             /* a CUDA runtime call failed (see nv4_last_cuda_error) */
#define NV4_ERR_DEVICE (-5)           /* current device is not an sm_100 GPU */

/* Activation layouts of nv4_rht_quant_pack. */
#define NV4_LAYOUT_BLOCK128 0 /* normalized 128-point WHT per K group (TP-local) */
#define NV4_LAYOUT_ROW_DH 1   /* row_DH_paley12_kron_sylvester_v1: H4096, or H12 (x) H1024 */

/* Flags of nv4_w4a4_grouped_gemm. */
#define NV4_GEMM_W_SCALE_GROUPED 1 /* w_scale is bf16 [N, K/128]; otherwise bf16 [N] */
#define NV4_GEMM_OUT_FP32 2        /* out is float32 [M, N] (diagnostic); otherwise bf16 */
#define NV4_GEMM_FORCE_STREAM 4    /* always use the weight-streaming mma.sync kernel (tests) */

/*
 * Randomized Hadamard transform, per-128-group activation quantisation and
 * INT4 packing.  Replaces nanovllm/kernels/rht_a4_tilelang.py:150-163
 * (rht_quant_pack) and its TileLang kernel (:19-136).
 *
 *   x          bf16 [m, k], 16-byte aligned
 *   signs      int8 [k], values +-1, 8-byte aligned
 *   out_packed int8 [m, k/2]: code of even k in the low nibble, 4-byte aligned
 *   out_scale  bf16 [m, k/128]: BF16 group scale, rounded before the codes
 *   layout     NV4_LAYOUT_BLOCK128 (k % 128 == 0) or NV4_LAYOUT_ROW_DH (k in {4096, 12288})
 *   clamp_lo   -7 (reference checkpoint contract) or -8 (full signed INT4 range)
 * code = round-half-even(x_rot / scale) clamped to [clamp_lo, 7]; an all-zero
 * group has scale 1.0; the scale floor is the BF16 tiny.
 */
int nv4_rht_quant_pack(const void* x, const void* signs, void* out_packed, void* out_scale, int64_t m,
                       int64_t k, int layout, int clamp_lo, void* stream);

/*
 * Same transform and quantisation as nv4_rht_quant_pack, but the codes are
 * written as GEMM-ready INT8 for nv4_w4a4_gemm_i8 instead of packed nibbles:
 *   out_codes int8 [m, k], 16-byte aligned; within every 32-wide K chunk the
 *             16 codes of even k come first (in k order), then the 16 of odd k.
 * The reference fuses nothing here; this is the first half of
 * nanovllm/layers/linear_w4a4.py:27-36 (W4A4Linear.forward) with the
 * intermediate in the layout the decode GEMM consumes without unpacking.
 */
int nv4_rht_quant_i8(const void* x, const void* signs, void* out_codes, void* out_scale, int64_t m, int64_t k,
                     int layout, int clamp_lo, void* stream);

/*
 * nv4_rht_quant_i8 of the down projection's input fused with its producer, the
 * MLP's SiluAndMul (nanovllm/layers/activation.py:8-11, nanovllm/models/qwen3.py
 * Qwen3MLP.forward): the source is the gate/up projection's output
 *   gate_up   bf16 [m, 2k] (gate in columns 0..k-1, up in k..2k-1), 16-byte aligned
 * and the prep input is h = bf16(silu(gate) * up), computed in FP32 with one
 * rounding at the end as the reference's compiled SiluAndMul does
 * (silu(g) = g / (1 + expf(-g)), IEEE division).  Outputs as nv4_rht_quant_i8
 * for the [m, k] input h, which is never written to memory.
 */
int nv4_silu_mul_rht_quant_i8(const void* gate_up, const void* signs, void* out_codes, void* out_scale, int64_t m,
                              int64_t k, int layout, int clamp_lo, void* stream);

/*
 * nv4_rht_quant_i8 of the QKV / gate-up input fused with its producer, the
 * decoder layer's residual add and RMSNorm (nanovllm/layers/layernorm.py:33-45
 * add_rms_forward; :17-27 rms_forward when residual is NULL):
 *   xf = f32(x) + f32(residual)                out_residual = bf16(xf)
 *   h  = bf16(bf16(xf * rsqrtf(mean(xf^2) + eps)) * weight)
 * then the prep of h (out_codes / out_scale as nv4_rht_quant_i8); h itself is
 * written to out_normed when that is non-NULL.  The sum of squares is taken in
 * a fixed order (deterministic; torch's order differs, so h can differ from
 * torch's in the last BF16 bit).  x, residual, out_residual, out_normed: bf16
 * [m, k]; weight: bf16 [k]; all 16-byte aligned.  Layouts: block128 with
 * k % 512 == 0 and k <= 16384, or row_DH with k == 4096.
 */
int nv4_add_rmsnorm_rht_quant_i8(const void* x, const void* residual, const void* weight, float eps,
                                  const void* signs, void* out_codes, void* out_scale, void* out_residual,
                                  void* out_normed, int64_t m, int64_t k, int layout, int clamp_lo, void* stream);

/*
 * Grouped INT4 GEMM: out[m, n] = sum_g fp32-FMA(dot_g(a, w), sa[m,g] * sw[n,g]),
 * groups of 128 along K in increasing g, one FP32 rounding per group, then BF16.
 * Replaces nanovllm/kernels/w4a4_grouped_kernel.py:104-129 (w4a4_grouped_gemm)
 * and, with NV4_GEMM_OUT_FP32, compile_grouped_gemm(..., output_fp32=True) (:31-91).
 *
 *   a_packed int8 [m, k/2] and w_packed int8 [n, k/2], 16-byte aligned rows (k % 32 == 0)
 *   a_scale  bf16 [m, k/128]
 *   w_scale  bf16 [n, k/128] with NV4_GEMM_W_SCALE_GROUPED, else bf16 [n]
 *            (per-channel: out = (sum_g fp32-FMA(dot_g, sa[m,g])) * sw[n])
 *   out      bf16 [m, n], or float32 with NV4_GEMM_OUT_FP32; every element is written
 * Requirements: m, n >= 1, k % 128 == 0, n % 8 == 0.
 */
int nv4_w4a4_grouped_gemm(const void* a_packed, const void* w_packed, const void* a_scale, const void* w_scale,
                          void* out, int64_t m, int64_t n, int64_t k, int flags, void* stream);

/*
 * The grouped GEMM with activations from nv4_rht_quant_i8 (int8 [m, k] in that
 * layout, 16-byte aligned) instead of packed nibbles; identical results.  The
 * second half of nanovllm/layers/linear_w4a4.py:27-36 (W4A4Linear.forward).
 */
int nv4_w4a4_gemm_i8(const void* a_codes, const void* w_packed, const void* a_scale, const void* w_scale, void* out,
                     int64_t m, int64_t n, int64_t k, int flags, void* stream);

/*
 * Diagnostic: exact per-group INT32 dot products dots[g, m, n] of the same
 * operands (the partials the GEMM scales and accumulates).  No reference
 * counterpart is exported; the reference checks these partials through its
 * FP32 diagnostic output (benchmarks/verify_w4a4_grouped.py:59-62).
 */
int nv4_w4a4_group_dots(const void* a_packed, const void* w_packed, int32_t* dots, int64_t m, int64_t n,
                        int64_t k, void* stream);

/*
 * GPTQ W4A16 dequant GEMM: out[m, n] = x[m, k] @ W[k, n], with
 * W[k, n] = bf16(bf16(w - z - 1) * bf16(scale[g, n])), g = k / group_size,
 * FP32 accumulation, BF16 output.  Replaces nanovllm/layers/linear_w4a16.py:11-59
 * (tl_dequant_matmul_w4a16); unlike the reference the caller's `out` need not
 * be zeroed and the split-K partials are summed in FP32.
 *
 *   x        bf16 [m, k]
 *   qweight  int32 [k/8, n]: nibble k%8 of k at bits 4*(k%8)
 *   qzeros   int32 [k/group_size, n/8]: nibble n%8 at bits 4*(n%8)
 *   scales   fp16 [k/group_size, n]
 *   out      bf16 [m, n]
 *   workspace   float32 scratch of nv4_w4a16_workspace_bytes(m, n, k) bytes
 *               (may be NULL when that size is 0).  Above 16 tokens it holds
 *               the FP32 partials of a K split (16-byte aligned, `out` 8-byte
 *               aligned); NULL or smaller there runs the GEMM unsplit.
 * Requirements: group_size == 128, k % 128 == 0, n % 64 == 0.
 */
int nv4_w4a16_gemm(const void* x, const void* qweight, const void* qzeros, const void* scales, void* out,
                   int64_t m, int64_t n, int64_t k, int64_t group_size, void* workspace, int64_t workspace_bytes,
                   void* stream);
int64_t nv4_w4a16_workspace_bytes(int64_t m, int64_t n, int64_t k);

/*
 * Which kernel nv4_w4a16_gemm runs for a shape, and its split, computed on the
 * host only (no GPU or CUDA call; sm_count is 148 on B200), assuming 16-byte
 * aligned operands and a workspace of nv4_w4a16_workspace_bytes.  No reference
 * counterpart: the reference launches one fixed configuration (BLOCK_M 16,
 * BLOCK_N 64, BLOCK_K 32, SPLIT_K 8; nanovllm/layers/linear_w4a16.py:138-146).
 * plan receives NV4_W4A16_PLAN_FIELDS int64 values, in order: kernel
 * (NV4_W4A16_KERNEL_*), K splits (cluster CTAs along K for the decode kernel,
 * K slices for the tcgen05 kernel, 1 = none), token tile, CTAs, workspace
 * bytes.  Returns NV4_OK, or NV4_ERR_INVALID_ARGUMENT for a shape or
 * sm_count nv4_w4a16_gemm would reject.
 */
#define NV4_W4A16_PLAN_FIELDS 5
#define NV4_W4A16_KERNEL_MMA 0    /* mma.sync tiles (shapes the others do not take) */
#define NV4_W4A16_KERNEL_DECODE 1 /* up to 16 tokens: TMA weight stream, cluster split-K */
#define NV4_W4A16_KERNEL_TC 2     /* more than 16 tokens: tcgen05, K split when tiles do not fill the SMs */
int nv4_w4a16_plan(int64_t m, int64_t n, int64_t k, int sm_count, int64_t* plan);

/*
 * nv4_w4a16_gemm without a workspace argument (no counterpart in the
 * reference, whose kernel adds into a pre-zeroed output instead).  Same
 * arguments, requirements and results as nv4_w4a16_gemm.
 *
 * Meant for callers that cannot hand out device memory at call time: a host
 * runtime that reserved all of HBM at start-up for its page pool and weights,
 * or a plain C caller with no device allocator of its own.  The call
 * allocates nothing: the split-K partial sums of small m go to a 2 MiB float32
 * array compiled into the library (one per device).
 *
 *   - Limit: when m <= 16 (the split-K case), m * n must not exceed
 *     NV4_W4A16_STATIC_SCRATCH_FLOATS; larger requests return
 *     NV4_ERR_UNSUPPORTED before anything is launched.  m > 16 needs no scratch.
 *   - Zero start: the split-K kernel adds into the first m * n floats of the
 *     array, so each call clears them on `stream` (cudaMemsetAsync) first.
 *   - Set-up: the first call on a device looks up the array's address with
 *     that device current (cudaGetSymbolAddress, which loads the library's
 *     kernels) and keeps it; make that first call before any stream capture.
 *   - Concurrency: every call on one device shares the one array.  Calls that
 *     may overlap (other streams, other host threads, without ordering between
 *     them) race on it and give wrong results; serialise them.
 */
#define NV4_W4A16_STATIC_SCRATCH_FLOATS (512 * 1024)
int nv4_w4a16_gemm_static(const void* x, const void* qweight, const void* qzeros, const void* scales, void* out,
                          int64_t m, int64_t n, int64_t k, int64_t group_size, void* stream);

/*
 * One-shot all-reduce of the row-parallel layers over NVLink peer memory (the
 * W4A4 counterpart of nanovllm/layers/linear.py:154-155, dist.all_reduce of
 * the partial outputs; the reference has no W4A4 tensor parallelism).
 *
 * Every rank allocates one peer buffer at set-up for outputs of up to
 * `capacity` elements: NV4_PEER_HEADER_BYTES of flags (zeroed), its FP32
 * partial [capacity] and the inboxes for the other ranks' partials.  The CUDA
 * IPC handles (NV4_IPC_HANDLE_BYTES each) are exchanged over the process
 * group and opened on the other ranks; one buffer serves every row-parallel
 * layer of the group.  Per call, the row-parallel GEMM writes its FP32 partial
 * at bufs[rank] + NV4_PEER_HEADER_BYTES, then nv4_peer_allreduce_bf16 copies
 * it into the peers' inboxes, waits for theirs, sums the partials in rank
 * order (identical results on all ranks) and writes BF16 [count] to `out`.
 * All ranks must make the same sequence of calls with the same counts; the
 * per-call synchronisation state lives in the buffers, so the calls may be
 * replayed from a CUDA graph.  A rank that does not arrive within 2 s makes
 * the others record an error (see nv4_device_error) and return.
 *
 *   bufs      world pointers: this rank's buffer at [rank], the opened peers' others
 *   world     2..8
 *   count     elements of this call, a multiple of 4, <= capacity
 *   capacity  the capacity every rank allocated with (a multiple of 4)
 */
#define NV4_PEER_HEADER_BYTES 16384
#define NV4_IPC_HANDLE_BYTES 64
#define NV4_PEER_MAX_TOKENS 32
int64_t nv4_peer_header_bytes(void);
int nv4_peer_buffer_alloc(int64_t capacity, void** buf, void* ipc_handle);
int nv4_peer_buffer_open(const void* ipc_handle, void** buf);
int nv4_peer_buffer_close(void* buf);  /* a buffer opened with nv4_peer_buffer_open */
int nv4_peer_buffer_free(void* buf);   /* a buffer from nv4_peer_buffer_alloc */
int nv4_peer_allreduce_bf16(void* const* bufs, int rank, int world, void* out, int64_t count, int64_t capacity,
                            void* stream);
/*
 * The row-parallel W4A4 GEMM and its all-reduce in two launches without the
 * FP32 partial round trip: the GEMM (GEMM-ready INT8 activation codes as in
 * nv4_w4a4_gemm_i8, up to NV4_PEER_MAX_TOKENS rows) stores each CTA's FP32
 * output tile straight into every rank's inbox over NVLink and releases one
 * flag per CTA on each peer; a second kernel waits for the peers' tiles and
 * sums them in rank order to BF16 [m, n] in `out` -- the same values as
 * nv4_w4a4_gemm_i8 (FP32) followed by nv4_peer_allreduce_bf16.  m * n must not
 * exceed `capacity`; flags: NV4_GEMM_W_SCALE_GROUPED only.  The two forms may
 * share one set of peer buffers; every rank makes the same sequence of calls.
 */
int nv4_w4a4_gemm_peer_allreduce_bf16(const void* a_codes, const void* w_packed, const void* a_scale,
                                      const void* w_scale, void* out, int64_t m, int64_t n, int64_t k, int flags,
                                      void* const* bufs, int rank, int world, int64_t capacity, void* stream);

/*
 * Launch plan of the decode (weight-streaming) GEMM that nv4_w4a4_gemm_i8 /
 * nv4_w4a4_grouped_gemm use for m <= 64 tokens, computed on the host only
 * (no GPU or CUDA call; sm_count is 148 on B200).  No reference counterpart:
 * the reference's TileLang configs (nanovllm/kernels/w4a4_grouped_kernel.py:
 * 21-28, 94-101) pick tile sizes from a JSON table instead.  peer != 0 plans
 * the fused row-parallel form (nv4_w4a4_gemm_peer_allreduce_bf16), whose grid
 * is limited to NV4_PEER_MAX_CTAS CTAs.  plan receives NV4_STREAM_PLAN_FIELDS
 * int32 values, in order: token tiles (8 tokens each) per CTA, 16-row weight
 * slabs per CTA, K-split warps per slab, token splits, token tiles per warp,
 * weight rows per CTA, ring stages, K stages (two groups each), shared memory
 * bytes, grid x, grid y, threads per CTA, producer warps.  The ring holds at
 * least min(K stages, K-split warps + producer warps) stages.  Returns NV4_OK,
 * or NV4_ERR_UNSUPPORTED for a shape the kernel cannot plan.
 */
#define NV4_STREAM_PLAN_FIELDS 13
#define NV4_PEER_MAX_CTAS 256
int nv4_w4a4_stream_plan(int64_t m, int64_t n, int64_t k, int flags, int sm_count, int peer, int32_t* plan);

/*
 * Decode attention over the paged BF16 KV cache of the end-to-end model:
 * replaces flash_attn_with_kvcache in nanovllm/layers/attention.py:71-73
 * (causal, one query token per sequence).
 *
 *   q             bf16 [batch, num_heads, head_dim] (the current token's queries)
 *   k_cache/v_cache  bf16 [pages, page_size, num_kv_heads, head_dim]
 *   block_tables  int32 [batch, max_pages]: page of each 256-token block
 *   context_lens  int32 [batch]: tokens of each sequence (including the current
 *                 one); 0 marks a padding row, whose output is zero
 *   out           bf16 [batch, num_heads, head_dim]
 *   workspace     nv4_paged_attention_workspace_bytes(batch, num_heads, max_pages) bytes
 * Query head h attends with KV head h / (num_heads / num_kv_heads) (grouped-
 * query attention, at most 8 query heads per KV head); softmax scale `scale`.
 * Requirements: head_dim == 128, page_size == 256.
 */
int64_t nv4_paged_attention_workspace_bytes(int64_t batch, int64_t num_heads, int64_t max_pages);
int nv4_paged_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* block_tables,
                               const int32_t* context_lens, void* out, void* workspace, int64_t workspace_bytes,
                               int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                               int64_t page_size, int64_t max_pages, float scale, void* stream);

/*
 * Per-head q/k RMSNorm, rotary embedding and KV-cache store of the fused QKV
 * projection output, one kernel (nanovllm/models/qwen3.py:87-92 q_norm /
 * k_norm / rotary_emb, and nanovllm/layers/attention.py:10-40 store_kvcache):
 *
 *   qkv        bf16 [tokens, (num_heads + 2 * num_kv_heads) * head_dim]: q | k | v
 *   q_weight, k_weight  bf16 [head_dim] RMSNorm weights; eps as the model's
 *   cos_sin    float32 [max_position, head_dim]: cos in the first half, sin in the second
 *   positions  int64 [tokens]
 *   slot_mapping int32 [tokens]: cache row (page * page_size + offset); < 0 stores nothing
 *   q_out      bf16 [tokens, num_heads, head_dim]
 *   k_out      bf16 [tokens, num_kv_heads, head_dim] or NULL (prefill attention input)
 *   k_cache/v_cache as nv4_paged_decode_attention (NULL with slot_mapping NULL: no store)
 * RMSNorm bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w); rotary on FP32 copies,
 * y1 = x1 cos - x2 sin, y2 = x2 cos + x1 sin, rounded to BF16.  head_dim == 128.
 */
int nv4_qk_norm_rope_store(const void* qkv, const void* q_weight, const void* k_weight, const float* cos_sin,
                           const int64_t* positions, const int32_t* slot_mapping, void* q_out, void* k_out,
                           void* k_cache, void* v_cache, int64_t tokens, int64_t num_heads, int64_t num_kv_heads,
                           int64_t head_dim, float eps, void* stream);

/* Library metadata and error reporting. */
int nv4_version(void);                      /* major*10000 + minor*100 + patch */
const char* nv4_status_string(int status);  /* static string for a status code */
int nv4_last_cuda_error(void);              /* cudaError_t of the last NV4_ERR_CUDA in this thread */
/* Reads and clears the error word that bounded device-side waits set when they
 * give up (0 = none).  Synchronises the current device. */
int nv4_device_error(int* code);

#ifdef __cplusplus
}
#endif

#endif /* NV4_H_ */
