/*
 * webpytorch_b200 — C ABI of the B200 (sm_100a) quantized-linear library (libqlinear.so).
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream passed as `void*`
 * (a cudaStream_t; NULL means the legacy default stream), runs asynchronously on that
 * stream, and returns an int status (QL_OK == 0). It never aborts and never frees what it
 * is given; the caller owns every buffer. On failure ql_last_error() returns a message for
 * the calling thread.
 *
 * Citations are to the reference project (xnetsc/webpytorch, package `webtorch`), whose
 * operator each entry point replaces.
 */
#ifndef WEBPYTORCH_B200_QLINEAR_H
#define WEBPYTORCH_B200_QLINEAR_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QL_API __attribute__((visibility("default")))
#else
#define QL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* element types of activations, scales and outputs */
enum { QL_F32 = 0, QL_F16 = 1, QL_BF16 = 2 };

/* status codes */
enum {
  QL_OK = 0,
  QL_ERR_ARG = 1,         /* bad size, null pointer or unsupported parameter combination */
  QL_ERR_ALIGN = 2,       /* a pointer or stride violates the alignment a kernel needs   */
  QL_ERR_UNSUPPORTED = 3, /* valid input this build does not implement                  */
  QL_ERR_CUDA = 4,        /* a CUDA runtime call failed (message says which)             */
  QL_ERR_TIMEOUT = 5      /* a bounded device-side wait gave up                           */
};

/* launch flags (bit set) for ql_set_launch_flags */
enum {
  /* Launch kernels as programmatic dependents of the previous kernel in the stream, so a
     GEMV streams its weights while the previous kernel is still finishing. Activations and
     outputs stay ordered; the previous kernel must not write this call's WEIGHTS. */
  QL_LAUNCH_PDL = 1
};

/* Library version as major*10000 + minor*100 + patch. */
QL_API int ql_version(void);

/* Message describing the last failure on the calling thread ("" if none). */
QL_API const char* ql_last_error(void);

/* Process-wide launch flags (QL_LAUNCH_*); returns the previous value. Default 0.
 * No counterpart in the reference (its WebGPU runtime batches dispatches itself,
 * src/webgpu/webgpuContext.ts:35,141-201). */
QL_API int ql_set_launch_flags(int flags);

/*
 * Exact GPTQ dequantisation to fp32, W[k, n] = scales[g, n] * (q[k, n] - (z[g, n] + zero_offset))
 * with g = g_idx[k] (or k / gs when g_idx is NULL), computed in double and rounded once to
 * fp32, so the result is bit-identical to the reference's numpy unpack.
 *   qweight int32 [K/per, N] (per = 32/bits values packed LSB-first along K)
 *   qzeros  int32 [K/gs, N/per] (packed LSB-first along N)
 *   scales  [K/gs, N] of scales_dtype (QL_F32 / QL_F16 / QL_BF16)
 *   W       fp32 [K, N]
 * Replaces: webtorch/_core.py:4046-4072 (_gptq_matmul_np's unpack) and
 *           webtorch/quantize.py:32-43 (dequant_int).
 */
QL_API int ql_gptq_dequant(const int32_t* qweight, const int32_t* qzeros, const void* scales,
                    int scales_dtype, const int32_t* g_idx, float* W, int K, int N, int gs,
                    int bits, float zero_offset, void* stream);

/*
 * Quantized linear y[M, N] = x[M, K] @ dequant(W) (+ bias), fp32 accumulation.
 *   x        [M, K] of x_dtype, row stride ldx (elements)
 *   x_perm   NULL, or int32 [K]: the kernel reads x[:, x_perm[k]] in place of x[:, k]
 *            (the activation-order permutation that goes with ql_gptq_sort_rows)
 *   qweight / qzeros / scales as in ql_gptq_dequant, group size gs (a multiple of 32)
 *   bias     NULL or fp32 [N]
 *   out      [M, N] of out_dtype, row stride ldo (elements)
 *   zero_offset 0 (reference's own packing) or 1 (AutoGPTQ "stores zero-1" convention)
 * Selects the kernel family from M: for small M a TMA-fed GEMV on the integer MMA (u8 weights
 * x s8 activation bytes, exact int32 group sums), for large M a tcgen05 dequant-GEMM.
 * Replaces: webtorch/_core.py:4008-4043 (_gptq_matmul), called from
 *           QuantizedLinear.forward webtorch/_core.py:4446-4456.
 */
QL_API int ql_gptq_matmul(const void* x, int x_dtype, long ldx, const int32_t* x_perm,
                   const int32_t* qweight, const int32_t* qzeros, const void* scales,
                   int scales_dtype, const float* bias, void* out, int out_dtype, long ldo,
                   int M, int K, int N, int gs, int bits, float zero_offset, void* stream);

/*
 * Bytes of device workspace ql_gptq_matmul_ws needs for an M x K activation: on the tensor-core
 * (large-M) path the fp16 staging of x plus one int per row, on the decode path (more than 4
 * tokens) the activations staged once as the integer MMA's operand.
 * No counterpart in the reference (its WebGPU buffers are allocated per call, _core.py:4022).
 */
QL_API size_t ql_gptq_matmul_workspace(int M, int K);

/*
 * ql_gptq_matmul with caller-provided device workspace (>= ql_gptq_matmul_workspace(M, K)
 * bytes, 256-byte aligned). Without it, ql_gptq_matmul takes the workspace from the
 * stream-ordered allocator (cudaMallocAsync) when the tensor-core path needs one.
 * Replaces: webtorch/_core.py:4008-4043 (_gptq_matmul), as ql_gptq_matmul.
 */
QL_API int ql_gptq_matmul_ws(const void* x, int x_dtype, long ldx, const int32_t* x_perm,
                             const int32_t* qweight, const int32_t* qzeros, const void* scales,
                             int scales_dtype, const float* bias, void* out, int out_dtype, long ldo,
                             int M, int K, int N, int gs, int bits, float zero_offset, void* workspace,
                             size_t workspace_bytes, void* stream);

/*
 * ql_gptq_matmul for callers that cannot allocate device memory at call time: hosts that hand
 * out all device memory through their own allocator or budget (inference servers, plugin
 * sandboxes, language bindings with no handle on a CUDA allocator) and code that must not
 * allocate under a latency budget. It allocates nothing. The large-M (tensor-core) path keeps
 * its scratch in a fixed 24 MiB device array inside the library, held by every GPU that loads
 * it until the process exits (ql_gptq_matmul_noalloc_max_scratch() returns the size); calls
 * whose M x K needs more than that fail with QL_ERR_UNSUPPORTED, and so does any call that would
 * otherwise reach the stream-ordered allocator. Every call looks up the array's device address
 * (which allocates nothing); the first lookup on a device may load the library's device code, so
 * make one call per device before any stream capture. All calls share the array: calls that can
 * overlap on the GPU (different streams) race and must be serialised by the caller. Calls of up
 * to 4 tokens use no scratch at all (decode calls of 5 to 63 tokens stage their activations there).
 * No counterpart in the reference.
 */
QL_API int ql_gptq_matmul_noalloc(const void* x, int x_dtype, long ldx, const int32_t* x_perm,
                                  const int32_t* qweight, const int32_t* qzeros, const void* scales,
                                  int scales_dtype, const float* bias, void* out, int out_dtype, long ldo,
                                  int M, int K, int N, int gs, int bits, float zero_offset, void* stream);

/* Bytes of the fixed scratch array ql_gptq_matmul_noalloc works in. No counterpart in the reference. */
QL_API size_t ql_gptq_matmul_noalloc_max_scratch(void);

/*
 * Synchronises the device and reports whether a tensor-core kernel gave up on a bounded
 * wait since the last call (QL_ERR_TIMEOUT), or a CUDA error is pending. Clears the flag.
 * No counterpart in the reference (its GPU calls have no device-side failure path).
 */
QL_API int ql_device_status(void);

/*
 * Load-time row sort for act-order (desc_act) checkpoints: qweight_out row k' takes packed
 * value k = perm[k'] of qweight_in (both int32 [K/per, N]). With perm = a stable argsort of
 * g_idx, every group becomes a contiguous run of gs rows and ql_gptq_matmul(x_perm = perm)
 * computes the same product as the unsorted weight with g_idx.
 * Replaces: nothing in the reference (it ignores g_idx: webtorch/_core.py:4056 and
 *           webtorch/llm.py:569-573); it is the loader-side half of desc_act support.
 */
QL_API int ql_gptq_sort_rows(const int32_t* qweight_in, const int32_t* perm, int32_t* qweight_out,
                      int K, int N, int bits, void* stream);

/*
 * Exact fp32 dequantisation of a GGUF Q4_K weight: W[n, k] for the [N, K] tensor stored as
 * N rows of K/256 super-blocks of 144 bytes (f16 d | f16 dmin | scales[12] | qs[128]).
 * value = (d*sc_j) * q - dmin*m_j with the products and the difference rounded like numpy.
 * Replaces: webtorch/ggufload.py:116-131,190-202 (dequant, Q4_K branch).
 */
QL_API int ql_q4k_dequant(const uint8_t* raw, float* W, int N, int K, void* stream);

/*
 * y[M, N] = x[M, K] @ W[N, K]^T (+ bias) with W decoded from the raw Q4_K bytes inside the
 * kernel (no load-time re-layout). x of x_dtype with row stride ldx; out of out_dtype with
 * row stride ldo; bias NULL or fp32 [N]. raw must be 16-byte aligned; K % 256 == 0. From 16
 * tokens on (N % 16 == 0) the call runs the tcgen05 GEMM, below that the decode GEMV.
 * Replaces: webtorch/_core.py:3720-3734 (ggml_matmul) with the Q4_K decode of
 *           _core.py:3061-3068,3116-3133, called from GGMLLinear.forward _core.py:4399-4406.
 */
QL_API int ql_q4k_matmul(const void* x, int x_dtype, long ldx, const uint8_t* raw, const float* bias,
                         void* out, int out_dtype, long ldo, int M, int K, int N, void* stream);

/* Bytes of device workspace ql_q4k_matmul_ws needs for M tokens of a K-input weight (calls of
 * more than 4 tokens stage their activations once in it, from 16 tokens on as the tensor-core
 * path's fp16 rows; 0 below 5 tokens).
 * No counterpart in the reference (its WebGPU buffers are allocated per call). */
QL_API size_t ql_q4k_matmul_workspace(int M, int K);

/* ql_q4k_matmul with caller-provided device workspace (>= ql_q4k_matmul_workspace(M, K) bytes,
 * 256-byte aligned); without it (or with too small a one) the staging comes from the
 * stream-ordered allocator.
 * Replaces: webtorch/_core.py:3720-3734 (ggml_matmul), as ql_q4k_matmul. */
QL_API int ql_q4k_matmul_ws(const void* x, int x_dtype, long ldx, const uint8_t* raw, const float* bias,
                            void* out, int out_dtype, long ldo, int M, int K, int N, void* workspace,
                            size_t workspace_bytes, void* stream);

/*
 * Exact fp32 dequantisation of a GGUF weight of ggml type Q8_0 (8), Q4_K (12), Q5_K (13) or
 * Q6_K (14): W[n, k] for the [N, K] tensor stored as N rows of K / block blocks, each value
 * rounded exactly as the reference's numpy expression ((d*sc)*q for Q6_K, d*q for Q8_0,
 * (d*sc*q) - (dmin*m) for Q4_K / Q5_K). K % 256 == 0.
 * Replaces: webtorch/ggufload.py:140-145,190-246 (dequant: Q8_0, Q4_K, Q5_K, Q6_K branches).
 */
QL_API int ql_ggml_dequant(int ggml_type, const uint8_t* raw, float* W, int N, int K, void* stream);

/*
 * y[M, N] = x[M, K] @ W[N, K]^T (+ bias) with W decoded from the GGUF bytes inside the kernel,
 * for ggml types Q8_0, Q4_K, Q5_K, Q6_K (the ids above; Q4_K goes to ql_q4k_matmul). Rows must
 * be 4-byte aligned (Q8_0: K % 64 == 0, Q6_K: K % 512 == 0). Other arguments as ql_q4k_matmul.
 * Replaces: webtorch/_core.py:3720-3734 (ggml_matmul) with the decode fragments of
 *           _core.py:3071-3177 dispatched by _GGML_TYPES (_core.py:3608-3638).
 */
QL_API int ql_ggml_matmul(const void* x, int x_dtype, long ldx, const uint8_t* raw, int ggml_type,
                          const float* bias, void* out, int out_dtype, long ldo, int M, int K, int N,
                          void* stream);

/*
 * GPTQ-format quantisation of a dense weight W (out = N rows of in = K values, of w_dtype, row
 * stride ldw) on the GPU: asymmetric min/max per group of gs input rows, zero-padded to
 * Kp = K rounded up to gs and Np = N rounded up to 32/bits. Writes qweight int32 [Kp/per, Np],
 * qzeros int32 [Kp/gs, Np/per] storing (zero point - zero_store_offset) (1: AutoGPTQ's zp - 1,
 * 0: the reference's own packing) and scales [Kp/gs, Np] (QL_F16 or QL_F32). Bit-identical to
 * the reference's float32 numpy quantiser.
 * Replaces: webtorch/quantize.py:80-106 (_quantize_raw, _pack_autogptq) and, with
 *           zero_store_offset 0, webtorch/_core.py:3782-3824 (_gptq_quantize) on float32 weights.
 */
QL_API int ql_gptq_quantize(const void* W, int w_dtype, long ldw, int N, int K, int gs, int bits,
                            int zero_store_offset, int32_t* qweight, int32_t* qzeros, void* scales,
                            int scales_dtype, void* stream);

/*
 * The quantized linear of a decode step with its neighbours fused in (decode path, M <= 16):
 *   a = x                                        (glu == 0, norm_weight == NULL)
 *   a = silu(x[:, :K]) * x[:, K:2K]              (glu == K: x rows hold [gate | up], ldx >= 2K)
 *   a = x / sqrt(mean(x^2) + norm_eps) * w       (norm_weight w [K] fp32: RMSNorm over each row)
 *   out = a @ dequant(W) + bias + residual       (bias, residual [M, ld_residual] fp32, optional)
 * residual may be the same buffer as out (each element is read and written by one thread).
 * The norm and SwiGLU prologues are applied while the activations are staged for the integer MMA
 * (no separate launch, no intermediate); arguments otherwise as ql_gptq_matmul_ws. M > 16 and
 * shapes outside the TMA-fed GEMV (N % 32, K % 128, group size) return QL_ERR_UNSUPPORTED.
 * Replaces: the decode step's `_rms` -> q/k/v / gate / up projections, `silu(gate) * up` -> down,
 *           and the residual adds (webtorch/lm_engine.py:62-64,84-87,89-107; llm.py:1591-1616).
 */
QL_API int ql_gptq_matmul_fused(const void* x, int x_dtype, long ldx, const int32_t* x_perm,
                                const int32_t* qweight, const int32_t* qzeros, const void* scales,
                                int scales_dtype, const float* bias, const float* norm_weight, float norm_eps,
                                int glu, const float* residual, long ld_residual, void* out, int out_dtype,
                                long ldo, int M, int K, int N, int gs, int bits, float zero_offset,
                                void* workspace, size_t workspace_bytes, void* stream);

/*
 * One decode position of grouped-query attention: qkv [1, (NH + 2 NKV) * HD] fp32 (q heads, then
 * k, then v), rotary tables rope_cos / rope_sin [lmax, HD/2] fp32, position pos[0] read on the
 * device (int32, so a captured graph replays for every token), caches kcache / vcache
 * [NKV, lmax, HD] fp32 (this position's rotated k and v are written), out [NH * HD] fp32 =
 * softmax(q_rot . K[0..pos]^T * scale) . V per head (key/value head h / (NH / NKV)). A position
 * outside 0 .. lmax - 1 writes NaN outputs and leaves the caches alone. lmax <= 8192; HD a
 * multiple of 8; caches 16-byte aligned. Positions are split over CTAs of 64; workspace (>= ql_decode_attention_workspace bytes, 256-byte aligned) holds their
 * partial results and one counter per head, which must be zero before the first call (the kernel
 * leaves them at zero). Calls that share a workspace must not overlap on the GPU.
 * Replaces: webtorch/lm_engine.py:66-74 (_rope, _rot) and the attention of _block
 *           (lm_engine.py:89-101) / _decode_fwd (llm.py:1596-1611) at one position.
 */
QL_API int ql_decode_attention(const float* qkv, int NH, int NKV, int HD, const float* rope_cos,
                               const float* rope_sin, const int32_t* pos, float* kcache, float* vcache, int lmax,
                               float scale, float* out, void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace ql_decode_attention needs for NH heads of HD over a cache of lmax positions.
 * No counterpart in the reference. */
QL_API size_t ql_decode_attention_workspace(int NH, int HD, int lmax);

/* ---------------------------------------------------------------------------------------
 * Mixture-of-experts block. Replaces the body of `moe_mlp` (webtorch/lm_engine.py:294-329):
 * the host-side softmax / argpartition / per-expert loop becomes device routing plus two
 * grouped GEMMs over expert-sorted rows, so a step needs no host round trip.
 *
 *   ql_moe_route           logits [T, E] fp32 -> topk_idx/topk_w [T, top_k] (softmax over all
 *                          experts, top_k by value, ties to the lower index; renormalised when
 *                          norm_topk_prob, as lm_engine.py:301-307), counts [E], offsets [E+1]
 *                          (expert e owns rows offsets[e] .. offsets[e+1]-1 of the P = T*top_k
 *                          sorted rows), the active-expert list, the tile table (tiles of
 *                          tile_rows rows, 2 ints each; max_tiles >= P/tile_rows + min(E, P)),
 *                          row_token [P] (token of each sorted row) and pair_row [T*top_k].
 *                          cursor [E] is scratch. E <= 1024, top_k <= 16.
 *   ql_moe_grouped_matmul  y[r] = x[row_token[r]] @ W_e (row_token NULL: x[r]) for every sorted
 *                          row r of expert e; W stacked [E] GPTQ packs (qweight [E][K/per][N],
 *                          qzeros [E][K/gs][N/per], scales [E][K/gs][N]). Rows per expert are
 *                          read on the device; max_rows_per_expert is a host bound (<= T) that
 *                          sizes the decode kernel. Workspace: ql_moe_grouped_workspace bytes.
 *   ql_moe_act             a [P, I] = silu(y[:, :I]) * y[:, I:] (gate|up fused, _core.py:502)
 *   ql_moe_combine         out[t] = sum_j topk_w[t, j] * z[pair_row[t, j]]
 *                          (+ g[t] * shared[t], g = sigmoid(shared_gate[t * ldg]) or 1;
 *                          lm_engine.py:318-328)
 * --------------------------------------------------------------------------------------- */
QL_API int ql_moe_route(const float* logits, int T, int E, int top_k, int norm_topk_prob, int tile_rows,
                        int32_t* topk_idx, float* topk_w, int32_t* counts, int32_t* offsets, int32_t* cursor,
                        int32_t* active, int32_t* n_active, int32_t* tiles, int32_t* n_tiles, int max_tiles,
                        int32_t* row_token, int32_t* pair_row, void* stream);

/* Grouping of n rows by given ids in [0, G) (the expert-parallel dispatch groups (token, k)
 * pairs by destination rank, the receiving rank groups its rows by local expert): counts, offsets
 * [G+1], active list, tile table as ql_moe_route; row_src[r] = the input row placed at sorted row
 * r, pos_of[i] = the sorted row of input row i. Replaces the host-side `np.where(topk_idx == e)`
 * gathers of lm_engine.py:311-316. */
QL_API int ql_moe_group(const int32_t* ids, int n, int G, int tile_rows, int32_t* counts, int32_t* offsets,
                        int32_t* cursor, int32_t* active, int32_t* n_active, int32_t* tiles, int32_t* n_tiles,
                        int max_tiles, int32_t* row_src, int32_t* pos_of, void* stream);

/* Tile height the grouped matmul expects in the routing tile table for P rows over E experts of
 * a K-input projection: 32, 64 or 128 when it takes the tensor-core GEMM (from the average rows
 * per active expert), else 4 or 8 (decode GEMV tiles: about twice the average rows per
 * active expert, at most the bound on rows per expert).
 * Pass it as ql_moe_route's tile_rows.
 * No counterpart in the reference. */
QL_API int ql_moe_tile_rows(long P, int E, int K, int gs, int max_rows_per_expert);

QL_API size_t ql_moe_grouped_workspace(long P, int E, int K, int gs);

QL_API int ql_moe_grouped_matmul(const void* x, int x_dtype, long ldx, const int32_t* row_token, long P,
                                 const int32_t* qweight, const int32_t* qzeros, const void* scales,
                                 int scales_dtype, int E, const int32_t* offsets, const int32_t* active,
                                 const int32_t* n_active, const int32_t* tiles, const int32_t* n_tiles,
                                 int max_tiles, int tile_rows, int max_rows_per_expert, void* out, int out_dtype,
                                 long ldo, int K, int N, int gs, int bits, float zero_offset, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* The down projection of the expert FFN straight from the fused gate|up output: out[p] =
 * (silu(y[p, :K]) * y[p, K:2K]) @ W_e, the activation formed while staging (no [P, K]
 * intermediate, no separate ql_moe_act launch), on every tile height: the decode GEMV stages
 * it per CTA, the tensor-core GEMM in its fp16 staging pass (the same workspace as
 * ql_moe_grouped_matmul, ql_moe_grouped_workspace(P, E, K, gs) bytes). The result is
 * bit-identical to ql_moe_act (fp32) followed by ql_moe_grouped_matmul.
 * Replaces: webtorch/lm_engine.py:317 (exp["down"](wt.silu(exp["gate"](xe)) * exp["up"](xe))). */
QL_API int ql_moe_grouped_matmul_swiglu(const void* y, int y_dtype, long ldy, long P, const int32_t* qweight,
                                        const int32_t* qzeros, const void* scales, int scales_dtype, int E,
                                        const int32_t* offsets, const int32_t* active, const int32_t* n_active,
                                        const int32_t* tiles, const int32_t* n_tiles, int max_tiles, int tile_rows,
                                        int max_rows_per_expert, void* out, int out_dtype, long ldo, int K, int N,
                                        int gs, int bits, float zero_offset, void* workspace,
                                        size_t workspace_bytes, void* stream);

QL_API int ql_moe_act(const float* y, long P, int I, void* a, int a_dtype, void* stream);

QL_API int ql_moe_combine(const float* z, const int32_t* pair_row, const float* topk_w, int T, int top_k, int H,
                          const float* shared, long lds, const float* shared_gate, long ldg, void* out,
                          int out_dtype, long ldo, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WEBPYTORCH_B200_QLINEAR_H */
