/*
 * moe_b200.h — C ABI of the B200 (sm_100a) mixture-of-experts FFN path.
 *
 * libmoe_b200.so replaces, behind plain C calls, the CPU hot path of the
 * llm.c engine (hoathienvu8x/llm.c): the router GEMM + softmax + top-k,
 * token-to-expert dispatch, the grouped Q8_0/Q4_0 SwiGLU expert products
 * and the weighted combine.  No PyTorch and no C++ types cross this
 * boundary: only pointers, sizes and a tensor struct whose layout equals
 * the reference's tensor_t.
 *
 * Threading: one caller thread at a time (the reference's own model code
 * is single-threaded).  The library owns one CUDA stream per device.
 * Errors: functions returning int return MOE_OK (0) or a negative
 * moe_status; moe_last_error() describes the last failure.  The void
 * drop-ins abort with a message, like the reference's asserts.
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOE_API __attribute__((visibility("default")))
#else
#define MOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ */
/* Tensor carrier                                                       */
/* ------------------------------------------------------------------ */

/* Same memory layout as the reference's tensor_t (tensor.h:19-31) in the
 * build the reference Makefile makes (FEATURES has -DQ8_DOT, so the two
 * scratch fields are present).  A caller holding a tensor_t* passes it
 * cast to moe_tensor_t*. */
typedef struct moe_tensor {
	float *data;          /* MOE_F32 payload                       */
	void *qdata;          /* quantized payload (GGUF block layout) */
	int type;             /* enum tensor_dtype                     */
	uint64_t totlen;
	uint64_t maxcap;
	uint64_t dim[4];
	uint32_t ndim;
	void *scratch;        /* reference's Q8_K scratch (unused here) */
	size_t scratch_size;
} moe_tensor_t;

/* enum tensor_dtype (tensor.h:10-17); Q5_K (4) is not supported.  The
 * K-quants (Q4_K, Q6_K) serve the MoE experts: a layer's qtype is one type,
 * or gate/up and down types as MOE_QTYPE2 (the reference's Q4_K_M files
 * keep some down matrices in Q6_K). */
enum { MOE_F32 = 0, MOE_Q8_0 = 1, MOE_Q4_0 = 2, MOE_Q4_K = 3, MOE_Q6_K = 5 };
#define MOE_QTYPE2(gate_up, down) ((gate_up) | ((down) << 8))
#define MOE_QTYPE_GU(t) ((t) & 0xFF)
#define MOE_QTYPE_DN(t) (((t) >> 8) & 0xFF ? ((t) >> 8) & 0xFF : (t) & 0xFF)

enum moe_status {
	MOE_OK = 0,
	MOE_ERR_INVALID = -1,     /* bad argument / shape          */
	MOE_ERR_UNSUPPORTED = -2, /* dtype or shape not handled    */
	MOE_ERR_CUDA = -3,        /* CUDA runtime error            */
	MOE_ERR_NOMEM = -4,       /* device allocation failed      */
	MOE_ERR_NOT_INIT = -5,    /* moe_init not called           */
	MOE_ERR_COMM = -6,        /* NCCL / expert-parallel error  */
	MOE_ERR_TIMEOUT = -7      /* bounded wait expired          */
};

/* flags for the layer entry points */
#define MOE_TOPK_EXACT  0x01 /* true top-k; default reproduces nn.c:276-308  */
#define MOE_DEVICE_IO   0x02 /* input/output pointers are device pointers    */
#define MOE_LANES_AVX2  0x04 /* router sums follow the AVX2 build (8 lanes); */
                             /* default follows the AVX-512 build (16 lanes) */
#define MOE_RENORM      0x08 /* Mixtral: renormalise the top-k weights       */
                             /* (llama.c:422-427); OLMoE does not            */
#define MOE_FORCE_GEMV  0x10 /* never use the prefill GEMM (T > 64): the    */
                             /* decode expert kernels for every batch size   */
#define MOE_FORCE_GEMM  0x20 /* use the prefill tcgen05 GEMM for any T (it  */
                             /* is the default above 64 tokens; fp16-rounded */
                             /* weights and activations: layer output about  */
                             /* 5e-4 rel-L2 from fp32)                       */
#define MOE_SIMPLE      0x80 /* use the plain CUDA-core expert kernels (the   */
                             /* cross-check path) instead of the MMA ones    */
#define MOE_PROFILE     0x40 /* record CUDA events between the layer's stages */
                             /* (read back with moe_layer_stage_ms)          */
#define MOE_NO_FUSE     0x100 /* decode-sized batches: use the five-launch   */
                             /* path instead of the fused layer kernel       */
#define MOE_EP_SHARDED  0x200 /* expert-parallel layers: x holds this rank's */
                             /* own tokens and out receives their outputs    */
                             /* (tokens travel to the experts' ranks and the */
                             /* rows back); see moe_layer_set_peers          */
#define MOE_NO_T1       0x400 /* one token: keep it on the fused layer kernel */
                             /* instead of the single-token expert GEMVs     */
#define MOE_FORCE_T1    0x800 /* one token: the single-token expert GEMVs for */
                             /* any expert type (default: Q4_0 experts)      */

/* ------------------------------------------------------------------ */
/* Library lifetime                                                     */
/* ------------------------------------------------------------------ */

/* Select CUDA device `device`, create the stream.  Idempotent. */
MOE_API int moe_init(int device);
/* Free every device buffer and registered weight; safe to call twice. */
MOE_API int moe_shutdown(void);
/* Text of the last error on this thread ("" if none). */
MOE_API const char *moe_last_error(void);
/* Library build/version string. */
MOE_API const char *moe_version(void);

/* ------------------------------------------------------------------ */
/* Weight residency                                                     */
/* ------------------------------------------------------------------ */

/* Upload a weight tensor (fp32 router or Q8_0/Q4_0 blocks, 1-3 dims) to
 * HBM once, keeping its GGUF byte layout.  Keyed by the host pointer
 * (qdata or data): any later call that passes this tensor, or a view into
 * it (tensor_at_q, olmoe.c:20-60), uses the device copy.  Unregistered
 * weights passed to a compute call are uploaded on first sight.
 * Replaces: nothing (the reference reads weights from the mmap'd GGUF,
 * gguf.c:490-530); this is the residency hook a caller adds after
 * gguf_tensor_3d (olmoe.c:180-182).
 * Lifetime rule: the device copy is trusted for as long as the host range
 * stays registered, as for the read-only GGUF mapping the reference uses.
 * A caller that frees or rewrites a registered host buffer must first call
 * moe_unregister_weights (or moe_shutdown). */
MOE_API int moe_register_weights(const moe_tensor_t *t);
MOE_API int moe_unregister_weights(const moe_tensor_t *t);
/* Bytes of weights resident on the current device. */
MOE_API size_t moe_resident_bytes(void);

/* ------------------------------------------------------------------ */
/* Same-signature drop-ins (host fp32 in/out, synchronous)              */
/* ------------------------------------------------------------------ */

/* Replaces tensor_mma_transposed_2x2 (matmul.h:30-31, matmul.c:451-462):
 * ret[m,n] = lhs[m,k] . rhs[n,k]^T (+ add), rhs fp32, Q8_0 or Q4_0.
 * lhs/ret/add are host fp32.  Aborts on error (the reference asserts). */
MOE_API void moe_tensor_mma_transposed_2x2(moe_tensor_t *ret, const moe_tensor_t *lhs,
				   const moe_tensor_t *rhs, const moe_tensor_t *add);
/* Same, returning a status instead of aborting. */
MOE_API int moe_tensor_mma_transposed_2x2_status(moe_tensor_t *ret, const moe_tensor_t *lhs,
					 const moe_tensor_t *rhs, const moe_tensor_t *add);

/* Replaces fused_ffn_silu (nn.h:35-39, nn.c:496-539): one token through a
 * SwiGLU FFN with quantized weights.  Returns 1 when done, 0 when not
 * applicable (in->dim[0] != 1 or fp32 weights), exactly like the
 * reference; aborts on a device error.  gate/up receive the gate and up
 * activations (gate holds silu(g)*u afterwards, as in the reference). */
MOE_API int moe_fused_ffn_silu(const moe_tensor_t *in, moe_tensor_t *out,
		       moe_tensor_t *gate, const moe_tensor_t *gate_w,
		       moe_tensor_t *up, const moe_tensor_t *up_w,
		       const moe_tensor_t *down_w);

/* ------------------------------------------------------------------ */
/* Layer entry points                                                   */
/* ------------------------------------------------------------------ */

/* The whole moe_ffn of olmoe.c:343-407 (or, with MOE_RENORM, the
 * Mixtral flavour of llama.c:393-457) in one call:
 *   input [T, d] fp32, output [T, d] fp32 (host, or device with
 *   MOE_DEVICE_IO); gate_inp [NE, d] fp32 router;
 *   gate_exps/up_exps [NE, d_ff, d] and down_exps [NE, d, d_ff]
 *   Q8_0/Q4_0 3-D tensors as gguf_tensor_3d returns them.
 * The caller's one-line change in moe_ffn is to call this instead. */
MOE_API int moe_ffn_forward(const moe_tensor_t *input, moe_tensor_t *output,
		    const moe_tensor_t *gate_inp, const moe_tensor_t *gate_exps,
		    const moe_tensor_t *up_exps, const moe_tensor_t *down_exps,
		    size_t topk, int flags);

/* Mixtral layout: per-expert 2-D tensors blk.L.ffn_{gate,up,down}.E.weight
 * (llama.c:157-166); arrays of n_experts pointers. */
MOE_API int moe_ffn_forward_split(const moe_tensor_t *input, moe_tensor_t *output,
			  const moe_tensor_t *gate_inp,
			  const moe_tensor_t *const *gate_exp,
			  const moe_tensor_t *const *up_exp,
			  const moe_tensor_t *const *down_exp,
			  size_t n_experts, size_t topk, int flags);

/* ------------------------------------------------------------------ */
/* Device-level API (plain device pointers; used by engines and tests)  */
/* ------------------------------------------------------------------ */

typedef struct moe_layer moe_layer; /* opaque */

typedef struct moe_layer_desc {
	int64_t d_model, d_ff, n_experts, top_k;
	int qtype;                   /* MOE_Q8_0, MOE_Q4_0; K-quants: Q4_K /
				      * Q6_K or MOE_QTYPE2 of them (CUDA-
				      * core GEMVs, one GPU)               */
	int flags;                   /* default flags for forward calls   */
	const float *router_w;       /* device [n_experts, d_model] fp32  */
	const float *router_bias;    /* device [n_experts] or NULL        */
	/* host arrays of n_experts DEVICE pointers to each expert's
	 * [d_ff,d] gate/up and [d,d_ff] down block matrices */
	const void *const *gate;
	const void *const *up;
	const void *const *down;
	/* expert parallelism: this rank computes experts
	 * [first_expert, first_expert + n_local); 0/0 means all */
	int64_t first_expert, n_local;
} moe_layer_desc;

MOE_API int moe_layer_create(moe_layer **out, const moe_layer_desc *desc);
MOE_API int moe_layer_destroy(moe_layer *layer);
/* out[T,d] = MoE(x[T,d]); x/out device fp32; stream = cudaStream_t or
 * NULL for the library stream.  Asynchronous: a failure inside the kernels
 * (an expired bounded wait, an expert id out of range) is recorded in the
 * layer's device error word, which stays set until moe_layer_status or
 * moe_layer_routing reads it. */
MOE_API int moe_layer_forward(moe_layer *layer, const float *x, float *out, int64_t T,
		      int flags, void *stream);
/* Waits for the device, then reads and clears the layer's error word:
 * MOE_OK, MOE_ERR_TIMEOUT (a bounded wait expired: a grid barrier, a
 * pipeline wait, or the expert-parallel exchange -- a rank missing or
 * behind) or MOE_ERR_INVALID (an expert id out of range; ranks that passed
 * different T to a token-sharded forward).  The output of the forward
 * that set it is not valid.  No counterpart in the reference, which
 * asserts (quant.c:571-574). */
MOE_API int moe_layer_status(moe_layer *layer);
/* Routing of the last forward, copied to HOST buffers (any may be NULL):
 * ids/weights [T,k] in top-k output order, counts [NE], offsets [NE+1],
 * perm [T*k] (pair p = t*k + slot, stably sorted by expert). */
MOE_API int moe_layer_routing(moe_layer *layer, int32_t *ids, float *weights, int32_t *counts,
		      int32_t *offsets, int32_t *perm);

/* Device time of each stage, summed over the MOE_PROFILE forwards since
 * the last call, in ms: [0] router logits (and the fp16 split of the
 * tokens), [1] softmax + top-k + dispatch, [2] gate/up + SwiGLU, [3] down,
 * [4] combine; [5] (if n >= 6) the number of forwards summed.  Five-launch
 * forwards are timed by CUDA events on the launching stream; the fused
 * decode kernel records %globaltimer at its phase boundaries (latest CTA
 * per boundary, grid barriers counted in the phase before them).
 * Synchronises the device and resets the sums. */
MOE_API int moe_layer_stage_ms(moe_layer *layer, float *ms, int n);

/* Expert parallelism over NVLink (no counterpart in the reference, which
 * runs on one host).  A layer created with n_local < n_experts owns an
 * exchange buffer; once every rank has passed its buffer's handle to the
 * others, decode-sized forwards (T <= 64) run the fused kernel on every
 * rank: the router and top-k run for all tokens on every rank (x must be
 * the same everywhere), each rank computes the (token, slot) rows of its
 * own experts and writes them into every rank's buffer as they are
 * produced, and every rank combines all rows in slot order -- so each
 * rank's output is the full layer output, identical on all ranks and to a
 * single GPU's.  Every rank must run the same sequence of forwards of the
 * layer.  Larger batches (and layers whose peers are not set) run the
 * router and top-k for all tokens and the grouped GEMMs for the local
 * experts; once moe_ep_init has been called, the ranks' partial outputs
 * (each the slot-order combine of its own experts' rows) are summed by an
 * NCCL all-reduce on the forward's stream, so every rank again ends with
 * the full output (identical on all ranks, within fp32 rounding of one
 * GPU's); without it the partial output is returned for the caller to sum.
 * moe_layer_ipc_handle writes this rank's 64-byte cudaIpcMemHandle_t;
 * moe_layer_set_peers takes all ranks' handles ([world][64] bytes, in rank
 * order), 2 <= world <= 8, once. */
MOE_API int moe_layer_ipc_handle(moe_layer *layer, void *handle);
MOE_API int moe_layer_set_peers(moe_layer *layer, int rank, int world, const void *handles);
/* Token-sharded expert parallelism (forward flag MOE_EP_SHARDED): every rank
 * passes its OWN T tokens (the same T on every rank) and receives their
 * outputs, as in data-parallel attention feeding expert-parallel FFNs.
 * Decode-sized forwards (T <= 64 and world*T*top_k <= 2048) run the fused
 * kernel: each rank writes its tokens (fp16 hi/lo) and top-k ids into every
 * rank's exchange buffer over NVLink, each rank's experts process the pairs
 * of all ranks' tokens, and each finished (token, slot) row goes straight to
 * the exchange buffer of the rank that owns the token, which combines its
 * tokens in slot order -- bit-identical to one GPU on the concatenated
 * batch.  Larger forwards (once moe_ep_init has been called) route the
 * token rows to the experts' ranks and the rows back with NCCL
 * point-to-point transfers (an all-to-all), with the grouped GEMMs between.
 * Every rank must run the same sequence of forwards with the same flags. */
/* Limit (ms) of the cross-rank waits of the fused kernel (default 2000). */
MOE_API int moe_layer_set_wait_ms(moe_layer *layer, int ms);
/* After an expired exchange wait: clear this rank's exchange counters and
 * error word.  Every rank calls it between two host-side barriers (so no
 * rank's next forward starts before every rank has reset) before the next
 * forward. */
MOE_API int moe_layer_ep_reset(moe_layer *layer);
/* The library's NCCL communicator for expert-parallel batches above 64
 * tokens (libnccl.so.2 is loaded at run time).  Rank 0 calls
 * moe_ep_unique_id (128 bytes) and shares the bytes out of band; then every
 * rank calls moe_ep_init(rank, world, id) once, after moe_init.
 * moe_ep_finalize (also run by moe_shutdown) destroys it. */
MOE_API int moe_ep_unique_id(void *id);
MOE_API int moe_ep_init(int rank, int world, const void *id);
MOE_API int moe_ep_finalize(void);

/* Diagnostics of the fused decode kernel: the raw %globaltimer stamps (ns)
 * of the latest MOE_PROFILE fused forward not yet consumed by
 * moe_layer_stage_ms, as [CTA][stamp] with 12 stamps per CTA: start, router
 * end, barrier 1 exit, top-k done, barrier 1b exit, dispatch done, routing
 * end, gate/up end, barrier 2 exit, down end, barrier 3 exit, end.  Returns the
 * number of values written (CTAs x 12) or a negative moe_status.  Has no
 * counterpart in the reference. */
MOE_API int moe_layer_phase_stamps(moe_layer *layer, uint64_t *out, int n);

/* y[m, rows] = x[m, cols] . W[rows, cols]^T with W in Q8_0/Q4_0 blocks on
 * the device (config-1 dense decode GEMV when m == 1).  Asynchronous. */
MOE_API int moe_gemv_device(const void *w, int qtype, int64_t rows, int64_t cols,
		    const float *x, int64_t m, float *y, void *stream);

/* No counterpart in the reference.  moe_gemv_device without any device
 * allocation, for callers that cannot allocate at the point of the call: a
 * real-time decode loop that must not take cudaMalloc's implicit
 * synchronisation, or an engine whose device memory budget is fixed and
 * handed out by someone else.  Inputs and outputs as for
 * moe_gemv_device (device pointers); the scratch (launch metadata and the
 * fp16 split of x) lives in one fixed 1 MiB device array inside the
 * library, so m * cols must not exceed 262080 (MOE_ERR_INVALID otherwise).
 * The array's device address is looked up on a device's first call: make
 * that call before any stream capture.  All calls share the array: calls
 * that overlap on the GPU (other streams or threads) race.  NULL stream =
 * the library stream (the first such call initialises the library on the
 * current device: a stream, no memory).  The call is asynchronous; a
 * bounded wait that expires inside it sets a sticky flag in the array,
 * which moe_sync reports as MOE_ERR_TIMEOUT (a caller on its own stream
 * synchronises that stream first). */
MOE_API int moe_gemv_device_noalloc(const void *w, int qtype, int64_t rows, int64_t cols,
				    const float *x, int64_t m, float *y, void *stream);

/* Synchronise the library stream.  Returns MOE_ERR_TIMEOUT (once) if a
 * moe_gemv_device_noalloc call on this device recorded an expired wait. */
MOE_API int moe_sync(void);

/* ------------------------------------------------------------------ */
/* Device memory helpers (so C callers need no CUDA headers)            */
/* ------------------------------------------------------------------ */
MOE_API void *moe_device_alloc(size_t bytes);
MOE_API int moe_device_free(void *p);
MOE_API int moe_memcpy_h2d(void *dst, const void *src, size_t bytes);
MOE_API int moe_memcpy_d2h(void *dst, const void *src, size_t bytes);
MOE_API void *moe_host_alloc(size_t bytes);     /* pinned */
MOE_API int moe_host_free(void *p);

/* Seeded synthetic inputs generated on the device (bench / tests).
 * Fills n values sd*N(0,1) of generator stream (seed, tag) starting at
 * element `offset`; same formula as the CPU generator.  And quantizes
 * rows*cols fp32 (device) into Q8_0/Q4_0 blocks (device) with the
 * reference quantizers' rounding rules. */
MOE_API int moe_synth_gauss(float *dst, uint64_t seed, uint64_t tag, uint64_t offset,
		    int64_t n, float sd, void *stream);
MOE_API int moe_quantize_device(const float *src, int64_t rows, int64_t cols, int qtype,
			void *dst, void *stream);

/* ------------------------------------------------------------------ */
/* Whole model on the device (OLMoE, llama / Mixtral)                   */
/* ------------------------------------------------------------------ */

/* Replaces the forward of models/olmoe/olmoe.c (olmoe_prefill /
 * olmoe_decode, olmoe.c:504-520) and models/llama/llama.c (llama_prefill /
 * llama_decode, llama.c:560-576): embedding, RMSNorm, Q/K/V projections,
 * QK-norm (OLMoE), RoPE, KV cache, causal attention (GQA for llama), output
 * projection, residuals, the MoE FFN layers of this library (or a dense
 * SwiGLU FFN), final norm, and lm_head.  The tensors are the GGUF views the
 * reference's loader makes (olmoe_load / llama_load: gguf_tensor_1d/2d/3d),
 * copied into HBM by moe_model_create; the model code keeps its own
 * loading and tokenizer. */
enum { MOE_ARCH_OLMOE = 0, MOE_ARCH_LLAMA = 1 };

typedef struct moe_model moe_model; /* opaque */

typedef struct moe_model_desc {
	int arch;                       /* MOE_ARCH_OLMOE or MOE_ARCH_LLAMA   */
	int64_t n_layers, d_model;
	int64_t n_heads, n_kv_heads;    /* OLMoE: n_kv_heads = n_heads        */
	int64_t head_len;               /* 128                                */
	int64_t vocab, context;
	int64_t n_experts, top_k, d_ff; /* n_experts 0: dense SwiGLU FFN      */
	float rope_theta;
	const moe_tensor_t *token_embd;  /* [vocab, d] F32/Q8_0/Q4_0          */
	const moe_tensor_t *output;      /* lm_head [vocab, d] Q8_0/Q4_0      */
	const moe_tensor_t *output_norm; /* [d] F32                           */
	/* arrays of n_layers tensors (attn_q_norm / attn_k_norm: OLMoE only,
	 * NULL arrays for llama; ffn_gate_inp: F32 router, MoE only) */
	const moe_tensor_t *const *attn_norm, *const *attn_q, *const *attn_k, *const *attn_v;
	const moe_tensor_t *const *attn_q_norm, *const *attn_k_norm, *const *attn_output;
	const moe_tensor_t *const *ffn_norm, *const *ffn_gate_inp;
	/* OLMoE: n_layers 3-D expert tensors [n_experts, d_ff, d] / [n_experts,
	 * d, d_ff]; llama with experts (Mixtral): n_layers * n_experts 2-D
	 * tensors, layer-major; dense llama: n_layers 2-D tensors */
	const moe_tensor_t *const *ffn_gate, *const *ffn_up, *const *ffn_down;
} moe_model_desc;

MOE_API int moe_model_create(moe_model **out, const moe_model_desc *desc);
MOE_API int moe_model_destroy(moe_model *m);
/* olmoe_prefill / llama_prefill: T tokens at positions pos (host arrays)
 * appended to the cache; output (host, may be NULL) receives the T
 * final-normed rows [T, d].  MOE_ERR_INVALID if the cache would overflow
 * (the reference only rotates in decode) or a position is outside
 * [0, context). */
MOE_API int moe_model_prefill(moe_model *m, const int *tok, const int *pos, size_t T,
			      float *output);
/* olmoe_decode / llama_decode: one token; the cache rotates (kvcache.c:
 * 29-55, keep context/2) when full, and positions past the context are
 * replaced by the cache size.  output (host, may be NULL): [d]. */
MOE_API int moe_model_decode(moe_model *m, int tok, int pos, float *output);
/* logits [vocab] (host) of row `row` of the last prefill/decode output:
 * tensor_mma_transposed_2x2(logits, row, output.weight) (olmoe.c:563) */
MOE_API int moe_model_logits(moe_model *m, size_t row, float *logits);
/* Greedy generation as olmoe_generate / llama_generate with --greedy
 * (olmoe.c:522-601, main.c:189-193): prefill the prompt at positions
 * pos.., pick the first maximum of the last row's logits, then decode the
 * pick and pick again, at most n times, stopping once a pick equals eos
 * (eos < 0: never).  The decode steps run as one CUDA graph replayed per
 * token.  tokens (host, n + 1 entries) receives the picks; returns their
 * number (>= 1) or an error status. */
MOE_API int moe_model_generate(moe_model *m, const int *prompt, size_t T, int n, int eos,
			       int *tokens);
/* device time (CUDA events on the model's stream) of the last
 * moe_model_generate: the prompt's prefill with the first pick, and the
 * decode steps with their picks (an eos check adds a host read per step) */
MOE_API int moe_model_timing(moe_model *m, float *prefill_ms, float *decode_ms);
/* empty the KV cache and reset the position (a new sequence) */
MOE_API int moe_model_reset(moe_model *m);
/* waits for the device; MOE_OK or the first error a kernel recorded since
 * the last call (MOE_ERR_INVALID: a token id outside the vocabulary, a
 * position or cache row out of range; MOE_ERR_TIMEOUT from a MoE layer) */
MOE_API int moe_model_status(moe_model *m);
/* how the decode step runs (bits): 1 a captured CUDA graph (once a decode
 * step has run), 2 the fused one-row kernels, 4 programmatic dependent
 * launches; or an error status */
MOE_API int moe_model_mode(moe_model *m);
/* the cache size and device bytes the model holds */
MOE_API int moe_model_info(moe_model *m, int64_t *cache_size, int64_t *pos, size_t *device_bytes);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H */
