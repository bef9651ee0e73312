/*
 * capi_harness.c -- TEST INFRASTRUCTURE ONLY: the C-side check of the
 * drop-in boundary.  oracle/Makefile compiles it against the reference's own
 * tensor.h (the -DQ8_DOT build the reference Makefile makes) and links it
 * with the reference's sources (ref_harness.c: ref_moe_ffn, the reference's
 * moe_ffn assembled from its public calls) and with libmoe_b200.so, into
 * oracle/_ref/capi_harness.
 *
 *  - At compile time: the reference's tensor_t and moe_tensor_t have the same
 *    size and field offsets (tensor.h:19-31), so a reference caller can pass
 *    its tensor_t pointers across the boundary.
 *  - At run time: the moe_ffn replacement of the integration patch for
 *    models/olmoe/olmoe.c:343-407 (the same body: one moe_ffn_forward call on
 *    the layer's tensor_t objects, built as gguf_tensor_3d builds them --
 *    qdata views, dim[0] outermost) or, with RENORM, the Mixtral patch for
 *    models/llama/llama.c:393-457 (per-expert 2-D tensors,
 *    moe_ffn_forward_split) runs on the same bytes as the reference's
 *    moe_ffn, and both outputs are written out.
 *
 * usage: capi_harness DIR T D F NE K QTYPE RENORM
 *   reads DIR/{x,router,gate,up,down}.bin (raw fp32 / GGUF blocks) and
 *   writes DIR/out_gpu.bin and DIR/out_ref.bin ([T][D] fp32)
 */
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "tensor.h"     /* the reference's */
#include "moe_b200.h"   /* this library's */

_Static_assert(sizeof(tensor_t) == sizeof(moe_tensor_t), "tensor_t size");
_Static_assert(offsetof(tensor_t, data) == offsetof(moe_tensor_t, data), "data");
_Static_assert(offsetof(tensor_t, qdata) == offsetof(moe_tensor_t, qdata), "qdata");
_Static_assert(offsetof(tensor_t, type) == offsetof(moe_tensor_t, type), "type");
_Static_assert(offsetof(tensor_t, totlen) == offsetof(moe_tensor_t, totlen), "totlen");
_Static_assert(offsetof(tensor_t, maxcap) == offsetof(moe_tensor_t, maxcap), "maxcap");
_Static_assert(offsetof(tensor_t, dim) == offsetof(moe_tensor_t, dim), "dim");
_Static_assert(offsetof(tensor_t, ndim) == offsetof(moe_tensor_t, ndim), "ndim");
_Static_assert(offsetof(tensor_t, scratch) == offsetof(moe_tensor_t, scratch), "scratch");
_Static_assert(offsetof(tensor_t, scratch_size) == offsetof(moe_tensor_t, scratch_size),
	       "scratch_size");
_Static_assert(TENSOR_F32 == MOE_F32 && TENSOR_Q8_0 == MOE_Q8_0 && TENSOR_Q4_0 == MOE_Q4_0,
	       "dtype enum");

int ref_moe_ffn(const float *x, size_t T, size_t d, const float *router_w, size_t NE,
		const float *router_bias, const void *gate, const void *up, const void *down,
		int qtype, size_t d_ff, size_t topk, int renorm, float *out, int32_t *ids_out,
		float *w_out);

static void *slurp(const char *dir, const char *name, size_t want)
{
	char path[4096];
	snprintf(path, sizeof(path), "%s/%s", dir, name);
	FILE *f = fopen(path, "rb");
	if (!f) {
		fprintf(stderr, "cannot open %s\n", path);
		_exit(2);
	}
	void *p = malloc(want ? want : 1);
	if (fread(p, 1, want, f) != want) {
		fprintf(stderr, "%s: short read\n", path);
		_exit(2);
	}
	fclose(f);
	return p;
}

static void spill(const char *dir, const char *name, const void *p, size_t n)
{
	char path[4096];
	snprintf(path, sizeof(path), "%s/%s", dir, name);
	FILE *f = fopen(path, "wb");
	if (!f || fwrite(p, 1, n, f) != n) {
		fprintf(stderr, "cannot write %s\n", path);
		_exit(2);
	}
	fclose(f);
}

/* a tensor_t view as gguf_tensor_{2,3}d makes it (tensor_reshape_3d:
 * dim[0] outermost, e.g. {NE, d_ff, d_model} for ffn_gate_exps) */
static tensor_t view(void *p, enum tensor_dtype type, int ndim, const uint64_t *dims)
{
	tensor_t t;
	memset(&t, 0, sizeof(t));
	if (type == TENSOR_F32)
		t.data = p;
	else
		t.qdata = p;
	t.type = type;
	t.ndim = (uint32_t)ndim;
	uint64_t n = 1;
	for (int i = 0; i < ndim; i++) {
		t.dim[i] = dims[i];
		n *= dims[i];
	}
	t.totlen = t.maxcap = n;
	return t;
}

/* ---- the integration patch's moe_ffn bodies ---- */
struct layer {
	tensor_t *gate_inp, *gate_exps, *up_exps, *down_exps;  /* OLMoE */
	tensor_t **gate_exp, **up_exp, **down_exp;             /* Mixtral */
};

static void moe_ffn_olmoe(struct layer *hl, tensor_t *input, tensor_t *output, size_t top_k)
{
	int rc = moe_ffn_forward((moe_tensor_t *)input, (moe_tensor_t *)output,
				 (moe_tensor_t *)hl->gate_inp, (moe_tensor_t *)hl->gate_exps,
				 (moe_tensor_t *)hl->up_exps, (moe_tensor_t *)hl->down_exps, top_k, 0);
	if (rc) {
		fprintf(stderr, "moe_ffn_forward: %s\n", moe_last_error());
		_exit(1);
	}
}

static void moe_ffn_mixtral(struct layer *hl, tensor_t *input, tensor_t *output, size_t n_exp,
			    size_t top_k)
{
	int rc = moe_ffn_forward_split((moe_tensor_t *)input, (moe_tensor_t *)output,
				       (moe_tensor_t *)hl->gate_inp,
				       (const moe_tensor_t *const *)hl->gate_exp,
				       (const moe_tensor_t *const *)hl->up_exp,
				       (const moe_tensor_t *const *)hl->down_exp, n_exp, top_k,
				       MOE_RENORM);
	if (rc) {
		fprintf(stderr, "moe_ffn_forward_split: %s\n", moe_last_error());
		_exit(1);
	}
}

int main(int argc, char **argv)
{
	if (argc != 9) {
		fprintf(stderr, "usage: %s DIR T D F NE K QTYPE RENORM\n", argv[0]);
		return 2;
	}
	const char *dir = argv[1];
	const size_t T = strtoull(argv[2], 0, 10), D = strtoull(argv[3], 0, 10);
	const size_t F = strtoull(argv[4], 0, 10), NE = strtoull(argv[5], 0, 10);
	const size_t K = strtoull(argv[6], 0, 10);
	const int qt = atoi(argv[7]), renorm = atoi(argv[8]);
	const size_t bb = qt == TENSOR_Q8_0 ? 34 : 18;
	const size_t gbytes = F * (D / 32) * bb, dbytes = D * (F / 32) * bb;
	float *x = slurp(dir, "x.bin", T * D * 4);
	float *wr = slurp(dir, "router.bin", NE * D * 4);
	uint8_t *g = slurp(dir, "gate.bin", NE * gbytes);
	uint8_t *u = slurp(dir, "up.bin", NE * gbytes);
	uint8_t *dn = slurp(dir, "down.bin", NE * dbytes);
	float *out_gpu = calloc(T * D, 4), *out_ref = calloc(T * D, 4);
	int32_t *ids = calloc(T * K, 4);
	float *wts = calloc(T * K, 4);

	const uint64_t dx[2] = {T, D}, dr[2] = {NE, D};
	tensor_t input = view(x, TENSOR_F32, 2, dx), output = view(out_gpu, TENSOR_F32, 2, dx);
	tensor_t router = view(wr, TENSOR_F32, 2, dr);
	struct layer hl = {&router, 0, 0, 0, 0, 0, 0};
	tensor_t ge, ue, de;
	tensor_t *gv = 0, *uv = 0, *dv = 0;
	tensor_t **gp = 0, **up = 0, **dp = 0;
	if (!renorm) {
		const uint64_t d3g[3] = {NE, F, D}, d3d[3] = {NE, D, F};
		ge = view(g, (enum tensor_dtype)qt, 3, d3g);
		ue = view(u, (enum tensor_dtype)qt, 3, d3g);
		de = view(dn, (enum tensor_dtype)qt, 3, d3d);
		hl.gate_exps = &ge, hl.up_exps = &ue, hl.down_exps = &de;
		moe_ffn_olmoe(&hl, &input, &output, K);
	} else {
		gv = calloc(NE, sizeof(tensor_t));
		uv = calloc(NE, sizeof(tensor_t));
		dv = calloc(NE, sizeof(tensor_t));
		gp = calloc(NE, sizeof(void *));
		up = calloc(NE, sizeof(void *));
		dp = calloc(NE, sizeof(void *));
		const uint64_t d2g[2] = {F, D}, d2d[2] = {D, F};
		for (size_t e = 0; e < NE; e++) {
			gv[e] = view(g + e * gbytes, (enum tensor_dtype)qt, 2, d2g);
			uv[e] = view(u + e * gbytes, (enum tensor_dtype)qt, 2, d2g);
			dv[e] = view(dn + e * dbytes, (enum tensor_dtype)qt, 2, d2d);
			gp[e] = &gv[e], up[e] = &uv[e], dp[e] = &dv[e];
		}
		hl.gate_exp = gp, hl.up_exp = up, hl.down_exp = dp;
		moe_ffn_mixtral(&hl, &input, &output, NE, K);
	}
	if (ref_moe_ffn(x, T, D, wr, NE, NULL, g, u, dn, qt, F, K, renorm, out_ref, ids, wts)) {
		fprintf(stderr, "ref_moe_ffn failed\n");
		_exit(1);
	}
	spill(dir, "out_gpu.bin", out_gpu, T * D * 4);
	spill(dir, "out_ref.bin", out_ref, T * D * 4);
	moe_shutdown();
	fflush(stdout);
	/* skip the reference's destructor (it joins its spinning workers) */
	_exit(0);
}
