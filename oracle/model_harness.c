/*
 * TEST INFRASTRUCTURE ONLY: the checker for the device model forward
 * (llm.c_b200 moe_model_*).  Never part of the product path.
 *
 * Drives the reference's own model code, compiled unmodified from its
 * sources (oracle/Makefile): gguf_load (gguf.c), olmoe_load/olmoe_prefill/
 * olmoe_decode (models/olmoe/olmoe.c:124,504,510) and llama_load/
 * llama_prefill/llama_decode (models/llama/llama.c:82,560,566).  The logits
 * are the reference's own lm_head product, tensor_mma_transposed_2x2 of one
 * output row with output.weight (olmoe.c:563,577, llama.c:628,643), taken
 * here from the same GGUF view the model loaded.
 *
 * Every call is plain C with host buffers, for ctypes in a child process
 * (loading the reference starts its spinning thread pool).
 */
#include "gguf.h"
#include "matmul.h"
#include "tensor.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* the models' entry points (models/olmoe/olmoe.h, models/llama/llama.h) */
struct olmoe;
struct llama;
void *olmoe_load(struct gguf *g);
void olmoe_prefill(struct olmoe *model, int *tok, int *pos, size_t T, tensor_t *output);
void olmoe_decode(struct olmoe *model, int tok, int pos, tensor_t *output);
void olmoe_close(void *ctx);
void *llama_load(struct gguf *g);
void llama_prefill(struct llama *model, int *tok, int *pos, size_t T, tensor_t *output);
void llama_decode(struct llama *model, int tok, int pos, tensor_t *output);
void llama_close(void *ctx);

struct refm {
	struct gguf *g;
	void *model;
	int llama;               /* 0: olmoe.c, 1: llama.c */
	size_t E, V, C;
	tensor_t *lm_head;       /* view of output.weight */
	tensor_t *out;           /* [C, E] model output rows */
	tensor_t *logits;        /* [V] */
};

void *refm_load(const char *path)
{
	struct refm *r = calloc(1, sizeof(*r));
	if (!r)
		return NULL;
	r->g = gguf_load(path);
	if (!r->g) {
		free(r);
		return NULL;
	}
	const char *arch = gguf_get_str(r->g, "general.architecture");
	r->llama = strcmp(arch, "olmoe") != 0;
	char key[64];
	snprintf(key, sizeof key, "%s.embedding_length", r->llama ? "llama" : "olmoe");
	r->E = gguf_get_uint32(r->g, key);
	snprintf(key, sizeof key, "%s.context_length", r->llama ? "llama" : "olmoe");
	r->C = gguf_get_uint32(r->g, key);
	r->V = gguf_get_arr_n(r->g, "tokenizer.ggml.tokens");
	r->model = r->llama ? llama_load(r->g) : olmoe_load(r->g);
	r->lm_head = gguf_tensor_2d(r->g, r->V, r->E, "output.weight");
	r->out = tensor_new_zero(2, r->C, r->E);
	r->logits = tensor_new_zero(1, r->V);
	return r;
}

/* output [T, E]: the final-normed hidden rows (olmoe.c:504, llama.c:560) */
int refm_prefill(void *h, const int *tok, const int *pos, size_t T, float *output)
{
	struct refm *r = h;
	if (T == 0 || T > r->C)
		return -1;
	int *tk = malloc(T * sizeof(int)), *ps = malloc(T * sizeof(int));
	memcpy(tk, tok, T * sizeof(int));
	memcpy(ps, pos, T * sizeof(int));
	if (r->llama)
		llama_prefill(r->model, tk, ps, T, r->out);
	else
		olmoe_prefill(r->model, tk, ps, T, r->out);
	memcpy(output, r->out->data, T * r->E * sizeof(float));
	free(tk);
	free(ps);
	return 0;
}

/* output [E] (olmoe.c:510, llama.c:566) */
int refm_decode(void *h, int tok, int pos, float *output)
{
	struct refm *r = h;
	if (r->llama)
		llama_decode(r->model, tok, pos, r->out);
	else
		olmoe_decode(r->model, tok, pos, r->out);
	memcpy(output, r->out->data, r->E * sizeof(float));
	return 0;
}

/* logits [V] = row [E] . output.weight^T */
int refm_logits(void *h, const float *row, float *logits)
{
	struct refm *r = h;
	tensor_t *x = tensor_new_zero(2, 1, r->E);
	memcpy(x->data, row, r->E * sizeof(float));
	tensor_reshape_1d(r->logits, r->V);
	tensor_mma_transposed_2x2(r->logits, x, r->lm_head, NULL);
	memcpy(logits, r->logits->data, r->V * sizeof(float));
	tensor_free(x);
	return 0;
}

void refm_close(void *h)
{
	struct refm *r = h;
	if (!r)
		return;
	if (r->llama)
		llama_close(r->model);
	else
		olmoe_close(r->model);
	tensor_free(r->out);
	tensor_free(r->logits);
	tensor_free_mapped(r->lm_head);
	gguf_close(r->g);
	free(r);
}
