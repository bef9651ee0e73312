/*
 * ref_harness.c — drives the UNMODIFIED reference sources (compiled from
 * where they lie by oracle/Makefile into oracle/_ref/) through their public
 * functions.  TEST INFRASTRUCTURE ONLY: it pins the oracle restatement and
 * gives the timed CPU baseline.  It is never linked into the product.
 *
 * moe_ffn is `static` in the reference (models/olmoe/olmoe.c:343-407,
 * models/llama/llama.c:393-457), as is tensor_at_q (olmoe.c:20-60), so the
 * layer is re-assembled here from the same public calls in the same order:
 * tensor_set, tensor_mma_transposed_2x2, softmax_1d, top_k, fused_ffn_silu,
 * tensor_div_scalar, tensor_add.
 */
#include "tensor.h"
#include "matmul.h"
#include "nn.h"
#include "quant.h"

#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static void view_2d(tensor_t *t, float *data, void *qdata, enum tensor_dtype type,
		    size_t rows, size_t cols)
{
	memset(t, 0, sizeof(*t));
	t->data = data;
	t->qdata = qdata;
	t->type = type;
	t->ndim = 2;
	t->dim[0] = rows;
	t->dim[1] = cols;
	t->totlen = rows * cols;
	t->maxcap = rows * cols;
}

static size_t qrow_bytes(int type, size_t cols)
{
	switch (type) {
	case TENSOR_Q8_0:
		return cols / 32 * sizeof(block_q8_0);
	case TENSOR_Q4_0:
		return cols / 32 * sizeof(block_q4_0);
	case TENSOR_Q4_K:
		return cols / QK_K * sizeof(block_q4_K);
	case TENSOR_Q6_K:
		return cols / QK_K * sizeof(block_q6_K);
	default:
		return cols * sizeof(float);
	}
}

/* a layer's weight types: gate/up in the low byte, down in the next byte
 * (0: the same) */
#define TYPE_GU(t) ((t) & 0xFF)
#define TYPE_DN(t) (((t) >> 8) & 0xFF ? ((t) >> 8) & 0xFF : (t) & 0xFF)

/* Same call sequence as moe_ffn.  Experts are 3-D [NE, rows, cols] tensors
 * (OLMoE) addressed like tensor_at_q; renorm = 1 adds the Mixtral weight
 * renormalisation (llama.c:422-427).  router_bias (may be NULL) is the
 * harness-level Zipf offset added between the router GEMM and the softmax. */
int ref_moe_ffn(const float *x, size_t T, size_t d, const float *router_w,
		size_t NE, const float *router_bias, const void *gate, const void *up,
		const void *down, int qtype, size_t d_ff, size_t topk, int renorm,
		float *out, int32_t *ids_out, float *w_out)
{
	if (topk > 64)
		return -1;
	tensor_t *input = tensor_new_zero(2, T, d);
	tensor_t *output = tensor_new_zero(2, T, d);
	tensor_t *logits = tensor_new_zero(2, T, NE);
	tensor_t *eg = tensor_new_zero(2, 1, d_ff);
	tensor_t *eu = tensor_new_zero(2, 1, d_ff);
	tensor_t *eo = tensor_new_zero(2, 1, d);
	tensor_t router;
	memcpy(input->data, x, T * d * sizeof(float));
	view_2d(&router, (float *)router_w, NULL, TENSOR_F32, NE, d);

	tensor_set(output, 0);
	tensor_mma_transposed_2x2(logits, input, &router, NULL);
	if (router_bias)
		for (size_t t = 0; t < T; t++)
			for (size_t e = 0; e < NE; e++)
				logits->data[t * NE + e] += router_bias[e];

	const int tg = TYPE_GU(qtype), td = TYPE_DN(qtype);
	size_t gsz = d_ff * qrow_bytes(tg, d);
	size_t dsz = d * qrow_bytes(td, d_ff);

	for (size_t t = 0; t < T; t++) {
		tensor_t tl;
		tensor_at(logits, t, &tl);
		softmax_1d(&tl);
		size_t ids[64];
		scalar_t w[64];
		top_k(&tl, ids, w, topk);
		if (renorm) {
			scalar_t sum = 0;
			for (size_t e = 0; e < topk; e++)
				sum += w[e];
			for (size_t e = 0; e < topk; e++)
				w[e] /= sum;
		}
		tensor_t tok_in;
		tensor_at(input, t, &tok_in);
		tensor_reshape_2d(&tok_in, 1, d);
		for (size_t e = 0; e < topk; e++) {
			tensor_t gw, uw, dw;
			view_2d(&gw, NULL, (char *)gate + ids[e] * gsz, tg, d_ff, d);
			view_2d(&uw, NULL, (char *)up + ids[e] * gsz, tg, d_ff, d);
			view_2d(&dw, NULL, (char *)down + ids[e] * dsz, td, d, d_ff);
			if (!fused_ffn_silu(&tok_in, eo, eg, &gw, eu, &uw, &dw)) {
				tensor_mma_transposed_2x2(eg, &tok_in, &gw, NULL);
				tensor_mma_transposed_2x2(eu, &tok_in, &uw, NULL);
				silu(eg);
				tensor_mul(eg, eg, eu);
				tensor_mma_transposed_2x2(eo, eg, &dw, NULL);
			}
			tensor_t tok_out;
			tensor_at(output, t, &tok_out);
			tensor_reshape_1d(eo, d);
			tensor_div_scalar(eo, eo, 1.0f / w[e]);
			tensor_add(&tok_out, &tok_out, eo);
			tensor_reshape_2d(eo, 1, d);
		}
		for (size_t e = 0; e < topk; e++) {
			if (ids_out)
				ids_out[t * topk + e] = (int32_t)ids[e];
			if (w_out)
				w_out[t * topk + e] = w[e];
		}
	}
	memcpy(out, output->data, T * d * sizeof(float));
	tensor_free(input);
	tensor_free(output);
	tensor_free(logits);
	tensor_free(eg);
	tensor_free(eu);
	tensor_free(eo);
	return 0;
}

/* C[m,n] = A[m,k] . B^T through tensor_mma_transposed_2x2 (matmul.h:30) */
void ref_gemm(const float *a, size_t m, size_t k, const void *b, int type, size_t n, float *c)
{
	tensor_t *lhs = tensor_new_zero(2, m, k);
	tensor_t *ret = tensor_new_zero(2, m, n);
	tensor_t rhs;
	memcpy(lhs->data, a, m * k * sizeof(float));
	if (type == TENSOR_F32)
		view_2d(&rhs, (float *)b, NULL, TENSOR_F32, n, k);
	else
		view_2d(&rhs, NULL, (void *)b, type, n, k);
	tensor_mma_transposed_2x2(ret, lhs, &rhs, NULL);
	memcpy(c, ret->data, m * n * sizeof(float));
	tensor_free(lhs);
	tensor_free(ret);
}

void ref_softmax(float *v, size_t n)
{
	tensor_t t;
	view_2d(&t, v, NULL, TENSOR_F32, n, 1);
	t.ndim = 1;
	t.dim[0] = n;
	softmax_1d(&t);
}

void ref_top_k(const float *v, size_t n, int32_t *ids, float *vals, size_t k)
{
	tensor_t t;
	size_t tmp[64];
	view_2d(&t, (float *)v, NULL, TENSOR_F32, n, 1);
	t.ndim = 1;
	t.dim[0] = n;
	top_k(&t, tmp, vals, k);
	for (size_t i = 0; i < k; i++)
		ids[i] = (int32_t)tmp[i];
}

void ref_quantize_row_q8_0(const float *x, void *y, size_t n)
{
	quantize_row_q8_0(x, (block_q8_0 *)y, n);
}

/* Q8_K activations (quant.c:627-654) and the integer K-quant dot against
 * them (quant.c:656-668 -> quant_avx2.h) */
void ref_quantize_row_q8K(const float *x, void *y, size_t n)
{
	quantize_row_q8(x, (block_q8_K *)y, n);
}

float ref_dot_q8K(const void *q8, const void *q, int type, size_t row, size_t n)
{
	return dot_q8_quant((const block_q8_K *)q8, NULL, q, type, row, n);
}

float ref_dot_f32_quant(const float *x, const void *q, int type, size_t row, size_t n)
{
	return dot_f32_quant(x, q, type, row, n);
}

void ref_dequant_row(const void *q, int type, size_t row, float *dst, size_t n)
{
	dequant_row(q, type, row, dst, n);
}

int ref_fused_ffn_silu(const float *x, size_t d, size_t d_ff, int type, const void *gw,
		       const void *uw, const void *dw, float *out)
{
	tensor_t *in = tensor_new_zero(2, 1, d);
	tensor_t *o = tensor_new_zero(2, 1, d);
	tensor_t *g = tensor_new_zero(2, 1, d_ff);
	tensor_t *u = tensor_new_zero(2, 1, d_ff);
	tensor_t tg, tu, td;
	memcpy(in->data, x, d * sizeof(float));
	view_2d(&tg, NULL, (void *)gw, TYPE_GU(type), d_ff, d);
	view_2d(&tu, NULL, (void *)uw, TYPE_GU(type), d_ff, d);
	view_2d(&td, NULL, (void *)dw, TYPE_DN(type), d, d_ff);
	int ok = fused_ffn_silu(in, o, g, &tg, u, &tu, &td);
	memcpy(out, o->data, d * sizeof(float));
	tensor_free(in);
	tensor_free(o);
	tensor_free(g);
	tensor_free(u);
	return ok;
}
