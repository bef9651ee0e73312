/*
 * oracle.h — CPU restatement of the llm.c mixture-of-experts FFN hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * B200 kernels in llm.c_b200/csrc.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference legs may load it.  The
 * product library never links, calls or falls back to it.
 *
 * Every routine restates the arithmetic of the reference C engine
 * (hoathienvu8x/llm.c), operation for operation, so that its results are
 * bit-identical to the reference built with -march=x86-64-v4 (AVX-512,
 * "lanes = 16") or -march=x86-64-v3 (AVX2, "lanes = 8").  The lane count
 * matters because the reference keeps one fp32 partial sum per SIMD lane
 * and reduces the lanes with a fixed butterfly at the end.
 *
 * Pinning: tests/test_oracle_kat.py checks this library against the
 * reference's own known-answer tests (test/nn.c, test/quant.c), and
 * tests/test_oracle_vs_ref.py against the reference sources compiled by
 * oracle/Makefile into oracle/_ref/ (bit-exact comparison).
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* tensor_dtype values of the reference (tensor.h:10-17) */
enum { ORC_F32 = 0, ORC_Q8_0 = 1, ORC_Q4_0 = 2, ORC_Q4_K = 3, ORC_Q6_K = 5 };
/* a layer's weight types: gate/up in the low byte, down in the next (0:
 * the same as gate/up) */
#define ORC_QTYPE_GU(t) ((t) & 0xFF)
#define ORC_QTYPE_DN(t) (((t) >> 8) & 0xFF ? ((t) >> 8) & 0xFF : (t) & 0xFF)

/* top-k selection rule */
enum {
	ORC_TOPK_REF = 0,   /* nn.c:276-308 exactly, index-0 seeding included */
	ORC_TOPK_EXACT = 1, /* true top-k by (value desc, index asc)          */
};

/* ---- synthetic input generator (shared with synth.cu) ----------------
 * stream = mix64(mix64(seed) ^ tag * 0xD1B54A32D192ED03); element i draws
 * two splitmix64 counters and one Box-Muller normal.  Tags: router 1,
 * gate 2, up 3, down 4, tokens 5, Zipf rank permutation 6, dense W 7,
 * dense x 8. */
uint64_t orc_mix64(uint64_t z);
uint64_t orc_stream_seed(uint64_t seed, uint64_t tag);
/* out[i] = sd * N(0,1) element (offset + i) of stream `stream` */
void orc_gauss(uint64_t stream, uint64_t offset, size_t n, float sd, float *out);
/* seeded permutation of 1..n (Fisher-Yates) -> Zipf logit bias
 * bias[e] = -s * ln(rank[e]) */
void orc_zipf_bias(uint64_t seed, size_t n, double s, float *bias);

/* ---- fp16 ------------------------------------------------------------ */
float orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_f16_rne(float f);   /* _cvtss_sh(f, 0): round to nearest even */
uint16_t orc_f32_to_f16_trunc(float f); /* test/quant.c:19-33 truncating variant  */

/* ---- quantizers ------------------------------------------------------ */
/* quant.c:62-78 (F16C build) */
void orc_quantize_row_q8_0(const float *x, void *blocks, size_t n);
/* test/quant.c:45-79 (the reference's only Q4_0 quantizer) */
void orc_quantize_row_q4_0(const float *x, void *blocks, size_t n);
/* quantize rows*cols floats row by row */
void orc_quantize_matrix(int type, const float *x, size_t rows, size_t cols, void *blocks);
size_t orc_row_bytes(int type, size_t cols);

/* ---- dot / dequant (quant.c:103-196, 577-614) ----------------------- */
void orc_dequant_row(const void *qdata, int type, size_t row, float *dst, size_t n);
float orc_dot_f32_quant(const float *x, const void *qdata, int type, size_t row,
			size_t n, int lanes);
float orc_dot_f32_f32(const float *x, const float *y, size_t n, int lanes);

/* ---- K-quants: Q8_K activations and the integer dots of the Q8_DOT build
 * (quant.c:627-668, quant_avx2.h), which both of the reference's x86 builds
 * select (__AVX2__) ---------------------------------------------------- */
/* sizeof(block_q8_K) = 4 + 256 + 32 */
#define ORC_Q8K_BYTES 292
void orc_quantize_row_q8K(const float *x, void *blocks, size_t n);
/* row `row` of a Q4_K / Q6_K matrix against Q8_K activations */
float orc_dot_q8K(const void *q8, const void *qdata, int type, size_t row, size_t n);

/* ---- router pieces --------------------------------------------------- */
/* logits[T,NE] = X[T,d] . Wr[NE,d]^T (matmul.c:91-131,169-245) */
void orc_router_logits(const float *x, size_t T, size_t d, const float *wr,
		       size_t NE, int lanes, float *logits);
void orc_softmax_1d(float *v, size_t n, int lanes);           /* nn.c:221-262 */
void orc_top_k(const float *v, size_t n, int32_t *ids, float *vals, size_t k,
	       int mode);                                       /* nn.c:276-308 */

/* stable counting sort of (token, slot) pairs by expert id.  Pair p =
 * t*k + slot.  counts[NE], offsets[NE+1], perm[T*k].  No reference
 * counterpart: the reference never groups tokens by expert. */
void orc_dispatch(const int32_t *ids, size_t T, size_t k, size_t NE,
		  int32_t *counts, int32_t *offsets, int32_t *perm);

/* ---- fused SwiGLU expert FFN for one token (nn.c:449-539) ------------ */
void orc_fused_ffn_silu(const float *x, size_t d, size_t d_ff, int type,
			const void *gate_w, const void *up_w, const void *down_w,
			int lanes, float *hidden /* [d_ff] */, float *out /* [d] */);

/* ---- dense quantized GEMM, C = A . B^T (matmul.c:270-324) ----------- */
void orc_gemm_q(const float *a, size_t m, size_t k, const void *b, int type,
		size_t n, int lanes, float *c);

/* ---- the MoE layer (olmoe.c:343-407, llama.c:393-457) --------------- */
typedef struct {
	size_t d_model, d_ff, n_experts, top_k;
	int qtype;      /* ORC_Q8_0 / ORC_Q4_0, or K-quants as ORC_QTYPE_GU / _DN */
	int renorm;     /* 1 = Mixtral renormalisation (llama.c:422-427) */
	int topk_mode;  /* ORC_TOPK_REF / ORC_TOPK_EXACT */
	int lanes;      /* 16 (AVX-512 build) or 8 (AVX2 build) */
	const float *router_w;   /* [NE, d] fp32 */
	const float *router_bias;/* [NE] or NULL (harness-level Zipf bias) */
	/* expert e's matrices: base + e * stride bytes (3-D tensors) */
	const void *gate, *up, *down;
	size_t gate_stride, up_stride, down_stride;
} orc_moe_layer;

/* out[T,d]; optional ids/weights[T,k] (after renorm), logits/probs[T,NE] */
void orc_moe_ffn(const orc_moe_layer *L, const float *x, size_t T, float *out,
		 int32_t *ids, float *weights, float *probs);
/* z[t*K + s] = y / (1 / w) for the slots whose expert is in [first, first +
 * nlocal) (other rows untouched); their sum over s, in slot order, is
 * orc_moe_ffn's output (the expert-parallel decomposition) */
void orc_moe_slot_terms(const orc_moe_layer *L, const float *x, size_t T, size_t first,
			size_t nlocal, float *z, int32_t *ids_out, float *w_out);

#ifdef __cplusplus
}
#endif
