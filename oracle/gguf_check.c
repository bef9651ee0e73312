/*
 * gguf_check.c -- TEST INFRASTRUCTURE ONLY: the reference's own GGUF loader
 * (gguf.c, compiled unmodified from the reference's sources by
 * oracle/Makefile into oracle/_ref/gguf_check) reading a file written by
 * llm.c_b200/gguf.py.  For every tensor it prints the reference's view of it
 * -- dtype and element count of the tensor_t that gguf_tensor_{1,2,3}d
 * return with the dims the model loaders ask for -- and an FNV-1a hash of
 * its bytes, plus the metadata the loaders read (olmoe.c:124-140,
 * llama.c:82-106).
 *
 * usage: gguf_check FILE.gguf
 */
#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <unistd.h>

#include "gguf.h"
#include "tensor.h"

/* gguf_close frees the tokenizer vocabulary (vocab.c), which is not built */
void vocab_free(struct gguf *g) { (void)g; }

static uint64_t fnv1a(const void *p, size_t n)
{
	const uint8_t *b = p;
	uint64_t h = 1469598103934665603ull;
	for (size_t i = 0; i < n; i++)
		h = (h ^ b[i]) * 1099511628211ull;
	return h;
}

static size_t bytes_of(const tensor_t *t)
{
	if (t->type == TENSOR_F32)
		return t->totlen * 4;
	return t->totlen / 32 * (t->type == TENSOR_Q8_0 ? 34 : 18);
}

static void show(const char *name, tensor_t *t)
{
	if (!t) {
		printf("%s missing\n", name);
		return;
	}
	const void *p = t->type == TENSOR_F32 ? (const void *)t->data : t->qdata;
	printf("%s %d %llu %016llx\n", name, (int)t->type, (unsigned long long)t->totlen,
	       (unsigned long long)fnv1a(p, bytes_of(t)));
}

int main(int argc, char **argv)
{
	if (argc != 2)
		return 2;
	struct gguf *g = gguf_load(argv[1]);
	if (!g)
		return 1;
	const char *arch = gguf_get_str(g, "general.architecture");
	char key[128];
	const int olmoe = strcmp(arch, "olmoe") == 0;
#define U32(k) (snprintf(key, sizeof(key), "%s." k, arch), gguf_get_uint32(g, key))
	const size_t E = U32("embedding_length"), L = U32("block_count");
	const size_t NE = U32("expert_count"), K = U32("expert_used_count");
	const size_t EI = U32("feed_forward_length"), H = U32("attention.head_count");
	const size_t KVH = olmoe ? H : U32("attention.head_count_kv");
	snprintf(key, sizeof(key), "%s.rope.freq_base", arch);
	const float theta = gguf_get_float32(g, key);
	const size_t V = gguf_get_arr_n(g, "tokenizer.ggml.tokens");
	printf("meta %s E=%zu L=%zu NE=%zu K=%zu EI=%zu H=%zu KVH=%zu V=%zu theta=%g\n", arch, E, L,
	       NE, K, EI, H, KVH, V, theta);
	const size_t HL = E / H;
	char name[128];
	show("token_embd.weight", gguf_tensor_2d(g, V, E, "token_embd.weight"));
	show("output.weight", gguf_tensor_2d(g, V, E, "output.weight"));
	show("output_norm.weight", gguf_tensor_1d(g, E, "output_norm.weight"));
	for (size_t i = 0; i < L; i++) {
#define T1(n) (snprintf(name, sizeof(name), "blk.%zu." n, i), show(name, gguf_tensor_1d(g, E, "%s", name)))
#define T2(n, a, b) (snprintf(name, sizeof(name), "blk.%zu." n, i), show(name, gguf_tensor_2d(g, a, b, "%s", name)))
		T1("attn_norm.weight");
		T2("attn_q.weight", H * HL, E);
		T2("attn_k.weight", KVH * HL, E);
		T2("attn_v.weight", KVH * HL, E);
		T2("attn_output.weight", E, H * HL);
		T1("ffn_norm.weight");
		T2("ffn_gate_inp.weight", NE, E);
		if (olmoe) {
			T1("attn_q_norm.weight");
			T1("attn_k_norm.weight");
			snprintf(name, sizeof(name), "blk.%zu.ffn_gate_exps.weight", i);
			show(name, gguf_tensor_3d(g, NE, EI, E, "%s", name));
			snprintf(name, sizeof(name), "blk.%zu.ffn_up_exps.weight", i);
			show(name, gguf_tensor_3d(g, NE, EI, E, "%s", name));
			snprintf(name, sizeof(name), "blk.%zu.ffn_down_exps.weight", i);
			show(name, gguf_tensor_3d(g, NE, E, EI, "%s", name));
		} else {
			for (size_t e = 0; e < NE; e++) {
				snprintf(name, sizeof(name), "blk.%zu.ffn_gate.%zu.weight", i, e);
				show(name, gguf_tensor_2d(g, EI, E, "%s", name));
				snprintf(name, sizeof(name), "blk.%zu.ffn_up.%zu.weight", i, e);
				show(name, gguf_tensor_2d(g, EI, E, "%s", name));
				snprintf(name, sizeof(name), "blk.%zu.ffn_down.%zu.weight", i, e);
				show(name, gguf_tensor_2d(g, E, EI, "%s", name));
			}
		}
	}
	fflush(stdout);
	_exit(0);
}
