/*
 * oracle.c — CPU restatement of the llm.c MoE FFN hot path (test only).
 *
 * TEST INFRASTRUCTURE: the parity checker for the CUDA kernels.  Nothing in
 * the product links or calls this file; see oracle.h for who may.
 *
 * The arithmetic follows the reference C sources line by line in *order of
 * floating-point operations* (which is what makes results bit-identical),
 * but the code is written from the description of that order, not copied.
 * Compile with -ffp-contract=off: every fused multiply-add below is an
 * explicit fmaf() standing for a _mm512_fmadd_ps / _mm256_fmadd_ps in the
 * reference, and no other contraction may happen.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define QK 32
#define GOLDEN 0x9E3779B97F4A7C15ULL

/* split [0, n) over the host's cores; used only by the input generator
 * and the quantizer, whose elements are independent */
struct par_job {
	void (*fn)(void *ctx, size_t lo, size_t hi);
	void *ctx;
	size_t lo, hi;
};

static void *par_run(void *p)
{
	struct par_job *j = p;
	j->fn(j->ctx, j->lo, j->hi);
	return NULL;
}

static void parallel_for(size_t n, size_t min_chunk, void (*fn)(void *, size_t, size_t), void *ctx)
{
	long nt = sysconf(_SC_NPROCESSORS_ONLN);
	if (nt < 1)
		nt = 1;
	if (nt > 32)
		nt = 32;
	if ((size_t)nt > n / min_chunk)
		nt = (long)(n / min_chunk);
	if (nt <= 1) {
		fn(ctx, 0, n);
		return;
	}
	pthread_t th[32];
	struct par_job jobs[32];
	for (long t = 0; t < nt; t++) {
		jobs[t] = (struct par_job){ fn, ctx, n * (size_t)t / (size_t)nt, n * (size_t)(t + 1) / (size_t)nt };
		pthread_create(&th[t], NULL, par_run, &jobs[t]);
	}
	for (long t = 0; t < nt; t++)
		pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------ */
/* generator: splitmix64 in counter form + Box-Muller                   */
/* ------------------------------------------------------------------ */

uint64_t orc_mix64(uint64_t z)
{
	z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
	z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
	return z ^ (z >> 31);
}

uint64_t orc_stream_seed(uint64_t seed, uint64_t tag)
{
	return orc_mix64(orc_mix64(seed) ^ (tag * 0xD1B54A32D192ED03ULL));
}

/* n-th draw (n >= 1) of the stream, mapped into the open interval (0,1) */
static double unit_draw(uint64_t stream, uint64_t n)
{
	uint64_t z = orc_mix64(stream + n * GOLDEN);
	return ((double)(z >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

struct gauss_ctx {
	uint64_t stream, offset;
	float sd;
	float *out;
};

static void gauss_range(void *p, size_t lo, size_t hi)
{
	struct gauss_ctx *c = p;
	for (size_t i = lo; i < hi; i++) {
		uint64_t e = c->offset + i;
		double u1 = unit_draw(c->stream, 2 * e + 1);
		double u2 = unit_draw(c->stream, 2 * e + 2);
		double g = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
		c->out[i] = (float)((double)c->sd * g);
	}
}

void orc_gauss(uint64_t stream, uint64_t offset, size_t n, float sd, float *out)
{
	struct gauss_ctx c = { stream, offset, sd, out };
	parallel_for(n, 1 << 16, gauss_range, &c);
}

void orc_zipf_bias(uint64_t seed, size_t n, double s, float *bias)
{
	uint64_t stream = orc_stream_seed(seed, 6);
	size_t *rank = malloc(n * sizeof(*rank));
	for (size_t i = 0; i < n; i++)
		rank[i] = i + 1;
	for (size_t i = n; i-- > 1;) {
		size_t j = (size_t)(orc_mix64(stream + (uint64_t)(n - i) * GOLDEN) % (i + 1));
		size_t t = rank[i];
		rank[i] = rank[j];
		rank[j] = t;
	}
	for (size_t e = 0; e < n; e++)
		bias[e] = (float)(-s * log((double)rank[e]));
	free(rank);
}

/* ------------------------------------------------------------------ */
/* fp16                                                                 */
/* ------------------------------------------------------------------ */

float orc_f16_to_f32(uint16_t h)
{
	uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
	uint32_t exp = (h >> 10) & 0x1f;
	uint32_t man = h & 0x3ff;
	uint32_t bits;
	if (exp == 0x1f) {
		bits = sign | 0x7f800000u | (man << 13);
	} else if (exp == 0) {
		if (man == 0) {
			bits = sign;
		} else {
			/* subnormal half: man * 2^-24, exact in fp32 */
			float v = (float)man * (1.0f / 16777216.0f);
			memcpy(&bits, &v, 4);
			bits |= sign;
		}
	} else {
		bits = sign | ((exp + 112) << 23) | (man << 13);
	}
	float f;
	memcpy(&f, &bits, 4);
	return f;
}

/* IEEE binary32 -> binary16, round to nearest even (what F16C's
 * _cvtss_sh(x, 0) does; quant.c:46-49). */
uint16_t orc_f32_to_f16_rne(float f)
{
	uint32_t x;
	memcpy(&x, &f, 4);
	uint32_t sign = (x >> 16) & 0x8000u;
	uint32_t ax = x & 0x7fffffffu;

	if (ax > 0x7f800000u)                 /* NaN: quiet, keep payload top */
		return (uint16_t)(sign | 0x7e00u | ((ax >> 13) & 0x3ffu));
	if (ax >= 0x477ff000u)                /* >= 65520 rounds to infinity */
		return (uint16_t)(sign | 0x7c00u);
	if (ax >= 0x38800000u) {              /* normal half */
		uint32_t r = ax - 0x38000000u;    /* rebias exponent by -112 */
		r += 0x0fffu + ((r >> 13) & 1u);
		return (uint16_t)(sign | (r >> 13));
	}
	uint32_t e = ax >> 23;
	if (e < 102)                          /* below 2^-25: rounds to zero */
		return (uint16_t)sign;
	uint32_t m = (ax & 0x7fffffu) | 0x800000u;
	uint32_t s = 126 - e;                 /* 14..24 */
	uint32_t q = m >> s;
	uint32_t rem = m & ((1u << s) - 1u);
	uint32_t half = 1u << (s - 1);
	if (rem > half || (rem == half && (q & 1u)))
		q++;
	return (uint16_t)(sign | q);
}

/* test/quant.c:19-33: truncating conversion used by the reference's test
 * quantizers (subnormals flush to signed zero). */
uint16_t orc_f32_to_f16_trunc(float f)
{
	uint32_t x;
	memcpy(&x, &f, 4);
	uint32_t sign = (x >> 16) & 0x8000u;
	uint32_t exp = (x >> 23) & 0xffu;
	uint32_t man = x & 0x7fffffu;
	if (exp == 0)
		return (uint16_t)sign;
	if (exp == 0xff)
		return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
	int e16 = (int)exp - 112;
	if (e16 >= 0x1f)
		return (uint16_t)(sign | 0x7c00u);
	if (e16 <= 0)
		return (uint16_t)sign;
	return (uint16_t)(sign | ((uint32_t)e16 << 10) | (man >> 13));
}

/* ------------------------------------------------------------------ */
/* quantizers                                                           */
/* ------------------------------------------------------------------ */

static void put_u16(uint8_t *p, uint16_t v)
{
	p[0] = (uint8_t)(v & 0xff);
	p[1] = (uint8_t)(v >> 8);
}

static uint16_t get_u16(const uint8_t *p)
{
	return (uint16_t)(p[0] | (p[1] << 8));
}

/* quant.c:62-78: d = amax/127 (stored as fp16, RNE), codes use 1/d in fp32 */
void orc_quantize_row_q8_0(const float *x, void *blocks, size_t n)
{
	uint8_t *out = blocks;
	for (size_t b = 0; b < n / QK; b++) {
		const float *xb = x + b * QK;
		float amax = 0.0f;
		for (int j = 0; j < QK; j++) {
			float a = fabsf(xb[j]);
			if (a > amax)
				amax = a;
		}
		float d = amax / 127.0f;
		float id = d != 0.0f ? 1.0f / d : 0.0f;
		uint8_t *blk = out + b * 34;
		put_u16(blk, orc_f32_to_f16_rne(d));
		for (int j = 0; j < QK; j++) {
			float p = xb[j] * id;
			blk[2 + j] = (uint8_t)(int8_t)roundf(p);
		}
	}
}

/* test/quant.c:45-79: d = amax/7 (fp16 by truncation); codes use 7/amax,
 * offset by 8 and clamped to 0..15; byte j holds element j (low nibble)
 * and element j+16 (high nibble). */
void orc_quantize_row_q4_0(const float *x, void *blocks, size_t n)
{
	uint8_t *out = blocks;
	for (size_t b = 0; b < n / QK; b++) {
		const float *xb = x + b * QK;
		float amax = 0.0f;
		for (int j = 0; j < QK; j++) {
			float a = fabsf(xb[j]);
			if (a > amax)
				amax = a;
		}
		float scale = amax / 7.0f;
		float inv = scale > 0.0f ? 7.0f / amax : 0.0f;
		uint8_t *blk = out + b * 18;
		put_u16(blk, orc_f32_to_f16_trunc(scale));
		for (int j = 0; j < QK / 2; j++) {
			float plo = xb[j] * inv;
			float phi = xb[j + QK / 2] * inv;
			int lo = (int)roundf(plo) + 8;
			int hi = (int)roundf(phi) + 8;
			lo = lo < 0 ? 0 : (lo > 15 ? 15 : lo);
			hi = hi < 0 ? 0 : (hi > 15 ? 15 : hi);
			blk[2 + j] = (uint8_t)(lo | (hi << 4));
		}
	}
}

size_t orc_row_bytes(int type, size_t cols)
{
	if (type == ORC_Q8_0)
		return cols / QK * 34;
	if (type == ORC_Q4_0)
		return cols / QK * 18;
	if (type == ORC_Q4_K)
		return cols / 256 * 144;
	if (type == ORC_Q6_K)
		return cols / 256 * 210;
	return cols * 4;
}

struct quant_ctx {
	int type;
	const float *x;
	size_t cols;
	uint8_t *blocks;
};

static void quant_range(void *p, size_t lo, size_t hi)
{
	struct quant_ctx *c = p;
	size_t rb = orc_row_bytes(c->type, c->cols);
	for (size_t r = lo; r < hi; r++) {
		if (c->type == ORC_Q8_0)
			orc_quantize_row_q8_0(c->x + r * c->cols, c->blocks + r * rb, c->cols);
		else
			orc_quantize_row_q4_0(c->x + r * c->cols, c->blocks + r * rb, c->cols);
	}
}

void orc_quantize_matrix(int type, const float *x, size_t rows, size_t cols, void *blocks)
{
	struct quant_ctx c = { type, x, cols, blocks };
	parallel_for(rows, 64, quant_range, &c);
}

/* ------------------------------------------------------------------ */
/* dot products with SIMD-lane partial sums                             */
/* ------------------------------------------------------------------ */

/* horizontal reduction of the reference's vector_reduce_sum
 * (vector_avx512.h:127-134, vector_avx2.h:130-136): halve the live lanes,
 * adding the upper half onto the lower, until one lane is left. */
static float lane_reduce(float *a, int lanes)
{
	for (int s = lanes / 2; s >= 1; s /= 2)
		for (int j = 0; j < s; j++)
			a[j] = a[j] + a[j + s];
	return a[0];
}

/* quant.c:103-124 */
static float dot_q8_0(const float *x, const uint8_t *row, size_t n, int lanes)
{
	float acc[16] = { 0 };
	for (size_t b = 0; b < n / QK; b++) {
		const uint8_t *blk = row + b * 34;
		float s = orc_f16_to_f32(get_u16(blk));
		for (int g = 0; g < QK; g += lanes)
			for (int j = 0; j < lanes; j++) {
				float q = (float)(int8_t)blk[2 + g + j];
				float sq = s * q;
				acc[j] = fmaf(sq, x[b * QK + g + j], acc[j]);
			}
	}
	return lane_reduce(acc, lanes);
}

/* quant.c:126-155 */
static float dot_q4_0(const float *x, const uint8_t *row, size_t n, int lanes)
{
	float acc[16] = { 0 };
	for (size_t b = 0; b < n / QK; b++) {
		const uint8_t *blk = row + b * 18;
		float s = orc_f16_to_f32(get_u16(blk));
		for (int g = 0; g < QK / 2; g += lanes)
			for (int j = 0; j < lanes; j++) {
				uint8_t byte = blk[2 + g + j];
				float lo = (float)((int)(byte & 15) - 8);
				float hi = (float)((int)(byte >> 4) - 8);
				float slo = s * lo;
				acc[j] = fmaf(slo, x[b * QK + g + j], acc[j]);
				float shi = s * hi;
				acc[j] = fmaf(shi, x[b * QK + g + j + QK / 2], acc[j]);
			}
	}
	return lane_reduce(acc, lanes);
}

/* ------------------------------------------------------------------ */
/* K-quants                                                             */
/* ------------------------------------------------------------------ */

/* get_scale_min_k4 (quant.h:62-71): 6-bit scale and min of sub-block j */
static void scale_min_k4(int j, const uint8_t *q, int *d, int *m)
{
	if (j < 4) {
		*d = q[j] & 63;
		*m = q[j + 4] & 63;
	} else {
		*d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
		*m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
	}
}

/* quant.c:200-236: element e of a Q4_K block, value (d*sc)*q - dmin*m with
 * the two products rounded, lanes of fused multiply-adds */
static float dot_q4_K(const float *x, const uint8_t *row, size_t n, int lanes)
{
	float acc[16] = { 0 };
	for (size_t b = 0; b < n / 256; b++) {
		const uint8_t *blk = row + b * 144;
		const float d = orc_f16_to_f32(get_u16(blk)), dmin = orc_f16_to_f32(get_u16(blk + 2));
		const uint8_t *sc = blk + 4, *q = blk + 16;
		for (int j = 0; j < 4; j++) {
			int s1, m1, s2, m2;
			scale_min_k4(2 * j, sc, &s1, &m1);
			scale_min_k4(2 * j + 1, sc, &s2, &m2);
			const float d1 = d * (float)s1, n1 = dmin * (float)m1;
			const float d2 = d * (float)s2, n2 = dmin * (float)m2;
			for (int k = 0; k < 32; k++) {
				const size_t e = b * 256 + j * 64 + k;
				const float v = d1 * (float)(q[j * 32 + k] & 15) - n1;
				acc[e % lanes] = fmaf(v, x[e], acc[e % lanes]);
			}
			for (int k = 0; k < 32; k++) {
				const size_t e = b * 256 + j * 64 + 32 + k;
				const float v = d2 * (float)(q[j * 32 + k] >> 4) - n2;
				acc[e % lanes] = fmaf(v, x[e], acc[e % lanes]);
			}
		}
	}
	return lane_reduce(acc, lanes);
}

/* Q6_K element e of a block: 6-bit value minus 32 (quant.c:305-410) and
 * its 8-bit scale */
static int q6_value(const uint8_t *blk, int e, int *scale)
{
	const int half = e / 128, r = e % 128, g = r / 32, k = r % 32;
	const uint8_t *ql = blk + half * 64, *qh = blk + 128 + half * 32;
	const int lo = g & 1 ? ql[32 + k] : ql[k];
	const int nib = g < 2 ? (lo & 15) : (lo >> 4);
	*scale = (int8_t)blk[192 + e / 16];
	return (nib | (((qh[k] >> (2 * g)) & 3) << 4)) - 32;
}

/* quant.c:305-410: (float)(q - 32) * (d * scale), lanes of fused
 * multiply-adds */
static float dot_q6_K(const float *x, const uint8_t *row, size_t n, int lanes)
{
	float acc[16] = { 0 };
	for (size_t b = 0; b < n / 256; b++) {
		const uint8_t *blk = row + b * 210;
		const float d = orc_f16_to_f32(get_u16(blk + 208));
		for (int e = 0; e < 256; e++) {
			int sc;
			const int q = q6_value(blk, e, &sc);
			const float v = (float)q * (d * (float)sc);
			const size_t i = b * 256 + e;
			acc[i % lanes] = fmaf(v, x[i], acc[i % lanes]);
		}
	}
	return lane_reduce(acc, lanes);
}

/* quant.c:627-654: per 256 values, the first value of largest magnitude
 * sets iscale = -127 / mval; q = min(127, roundf(iscale * x)); d = 1 /
 * iscale; bsums over each 16 */
void orc_quantize_row_q8K(const float *x, void *blocks, size_t n)
{
	uint8_t *out = blocks;
	for (size_t i = 0; i < n / 256; i++) {
		const float *xb = x + i * 256;
		uint8_t *y = out + i * ORC_Q8K_BYTES;
		float amax = 0.0f, mval = 0.0f;
		for (int j = 0; j < 256; j++) {
			const float a = fabsf(xb[j]);
			if (a > amax) {
				amax = a;
				mval = xb[j];
			}
		}
		memset(y, 0, ORC_Q8K_BYTES);
		if (amax == 0.0f)
			continue;
		const float iscale = -127.0f / mval;
		const float d = 1.0f / iscale;
		memcpy(y, &d, 4);
		int8_t *qs = (int8_t *)(y + 4);
		for (int j = 0; j < 256; j++) {
			const int v = (int)roundf(iscale * xb[j]);
			qs[j] = (int8_t)(v < 127 ? v : 127);
		}
		for (int j = 0; j < 16; j++) {
			int16_t s = 0;
			for (int k = 0; k < 16; k++)
				s = (int16_t)(s + qs[j * 16 + k]);
			memcpy(y + 260 + 2 * j, &s, 2);
		}
	}
}

/* quant_avx2.h: the integer sums are exact; per block acc += d * S (and,
 * for Q4_K, acc_m += dmin * M with M = sum_s m_s * (bsum_2s + bsum_2s+1),
 * added after the blocks), d = d8 * d_block, dmin = -d8 * dmin_block.  The
 * reference build contracts `acc += d * S` into a fused multiply-add. */
float orc_dot_q8K(const void *q8, const void *qdata, int type, size_t row, size_t n)
{
	const uint8_t *base = (const uint8_t *)qdata + row * orc_row_bytes(type, n);
	const uint8_t *y8 = q8;
	float acc = 0.0f, acc_m = 0.0f;
	for (size_t b = 0; b < n / 256; b++) {
		const uint8_t *y = y8 + b * ORC_Q8K_BYTES;
		float d8;
		memcpy(&d8, y, 4);
		const int8_t *qs = (const int8_t *)(y + 4);
		int16_t bs[16];
		memcpy(bs, y + 260, 32);
		if (type == ORC_Q4_K) {
			const uint8_t *blk = base + b * 144;
			const float d = d8 * orc_f16_to_f32(get_u16(blk));
			const float dmin = -d8 * orc_f16_to_f32(get_u16(blk + 2));
			int S = 0, M = 0;
			for (int s = 0; s < 8; s++) {
				int sc, m;
				scale_min_k4(s, blk + 4, &sc, &m);
				M += m * (bs[2 * s] + bs[2 * s + 1]);
				int t = 0;
				const int j = s / 2, hi = s & 1;
				for (int k = 0; k < 32; k++) {
					const int q = hi ? blk[16 + j * 32 + k] >> 4 : blk[16 + j * 32 + k] & 15;
					t += q * qs[s * 32 + k];
				}
				S += sc * t;
			}
			acc_m = fmaf(dmin, (float)M, acc_m);
			acc = fmaf(d, (float)S, acc);
		} else {
			const uint8_t *blk = base + b * 210;
			const float d = d8 * orc_f16_to_f32(get_u16(blk + 208));
			int S = 0;
			for (int e = 0; e < 256; e++) {
				int sc;
				const int q = q6_value(blk, e, &sc);
				S += sc * q * qs[e];
			}
			acc = fmaf(d, (float)S, acc);
		}
	}
	return acc + acc_m;
}

float orc_dot_f32_quant(const float *x, const void *qdata, int type, size_t row,
			size_t n, int lanes)
{
	const uint8_t *base = (const uint8_t *)qdata + row * orc_row_bytes(type, n);
	if (type == ORC_Q8_0)
		return dot_q8_0(x, base, n, lanes);
	if (type == ORC_Q4_K)
		return dot_q4_K(x, base, n, lanes);
	if (type == ORC_Q6_K)
		return dot_q6_K(x, base, n, lanes);
	return dot_q4_0(x, base, n, lanes);
}

/* quant.c:157-196 */
void orc_dequant_row(const void *qdata, int type, size_t row, float *dst, size_t n)
{
	const uint8_t *base = (const uint8_t *)qdata + row * orc_row_bytes(type, n);
	for (size_t b = 0; b < n / QK; b++) {
		if (type == ORC_Q8_0) {
			const uint8_t *blk = base + b * 34;
			float s = orc_f16_to_f32(get_u16(blk));
			for (int j = 0; j < QK; j++)
				dst[b * QK + j] = s * (float)(int8_t)blk[2 + j];
		} else {
			const uint8_t *blk = base + b * 18;
			float s = orc_f16_to_f32(get_u16(blk));
			for (int j = 0; j < QK / 2; j++) {
				dst[b * QK + j] = s * (float)((int)(blk[2 + j] & 15) - 8);
				dst[b * QK + j + QK / 2] = s * (float)((int)(blk[2 + j] >> 4) - 8);
			}
		}
	}
}

/* matmul.c:91-105.  The scalar tail is `sum += x*y`, which gcc contracts
 * into a fused multiply-add at -O3 on an FMA target. */
float orc_dot_f32_f32(const float *x, const float *y, size_t n, int lanes)
{
	float acc[16] = { 0 };
	size_t nv = n - n % (size_t)lanes;
	for (size_t i = 0; i < nv; i += (size_t)lanes)
		for (int j = 0; j < lanes; j++)
			acc[j] = fmaf(x[i + j], y[i + j], acc[j]);
	float sum = lane_reduce(acc, lanes);
	for (size_t i = nv; i < n; i++)
		sum = fmaf(x[i], y[i], sum);
	return sum;
}

/* ------------------------------------------------------------------ */
/* router                                                               */
/* ------------------------------------------------------------------ */

/* matmul.c:13-33 zeroes the result, then :107-131 (m == 1) or :169-245
 * (m > 1, fp32 rhs) add one lane-reduced dot product per element; both
 * paths use the same per-lane FMA chain. */
void orc_router_logits(const float *x, size_t T, size_t d, const float *wr,
		       size_t NE, int lanes, float *logits)
{
	for (size_t t = 0; t < T; t++)
		for (size_t e = 0; e < NE; e++)
			logits[t * NE + e] = 0.0f + orc_dot_f32_f32(x + t * d, wr + e * d, d, lanes);
}

/* nn.c:221-262 with tensor_max (tensor.c:479-517) */
void orc_softmax_1d(float *v, size_t n, int lanes)
{
	float mx = v[0];
	for (size_t i = 1; i < n; i++)
		if (v[i] > mx)
			mx = v[i];

	float lsum[16] = { 0 };
	size_t nv = n - n % (size_t)lanes;
	for (size_t i = 0; i < nv; i += (size_t)lanes)
		for (int j = 0; j < lanes; j++) {
			float e = expf(v[i + j] - mx);
			v[i + j] = e;
			lsum[j] = lsum[j] + e;
		}
	float sum = lane_reduce(lsum, lanes);
	for (size_t i = nv; i < n; i++) {
		v[i] = expf(v[i] - mx);
		sum = sum + v[i];
	}
	for (size_t i = 0; i < n; i++)
		v[i] = v[i] / sum;
}

/* nn.c:276-308.  The reference keeps k (index, value) slots sorted by
 * ascending value, all seeded with element 0, and admits a later element
 * only when it is strictly greater than the smallest slot; the newcomer
 * goes below any equal values already held.  Equivalently: rank the
 * sequence [v0 x k copies, v1, v2, ...] by (value desc, position asc) and
 * keep the first k, written out in ascending order. */
void orc_top_k(const float *v, size_t n, int32_t *ids, float *vals, size_t k, int mode)
{
	if (mode == ORC_TOPK_REF) {
		for (size_t s = 0; s < k; s++) {
			ids[s] = 0;
			vals[s] = v[0];
		}
		for (size_t i = 1; i < n; i++) {
			float nv = v[i];
			/* highest slot whose value is strictly below the newcomer */
			long pos = -1;
			for (size_t s = 0; s < k; s++)
				if (nv > vals[s])
					pos = (long)s;
			if (pos < 0)
				continue;
			for (long s = 0; s < pos; s++) {
				ids[s] = ids[s + 1];
				vals[s] = vals[s + 1];
			}
			ids[pos] = (int32_t)i;
			vals[pos] = nv;
		}
		return;
	}
	/* exact: element i outranks j if v_i > v_j, or equal and i < j */
	for (size_t i = 0; i < n; i++) {
		size_t rank = 0;
		for (size_t j = 0; j < n; j++)
			if (v[j] > v[i] || (v[j] == v[i] && j < i))
				rank++;
		if (rank < k) {
			ids[k - 1 - rank] = (int32_t)i;
			vals[k - 1 - rank] = v[i];
		}
	}
}

void orc_dispatch(const int32_t *ids, size_t T, size_t k, size_t NE,
		  int32_t *counts, int32_t *offsets, int32_t *perm)
{
	memset(counts, 0, NE * sizeof(*counts));
	for (size_t p = 0; p < T * k; p++)
		counts[ids[p]]++;
	offsets[0] = 0;
	for (size_t e = 0; e < NE; e++)
		offsets[e + 1] = offsets[e] + counts[e];
	int32_t *fill = malloc(NE * sizeof(*fill));
	memcpy(fill, offsets, NE * sizeof(*fill));
	for (size_t p = 0; p < T * k; p++)
		perm[fill[ids[p]]++] = (int32_t)p;
	free(fill);
}

/* ------------------------------------------------------------------ */
/* expert FFN                                                           */
/* ------------------------------------------------------------------ */

/* nn.c:449-539 (fused_ffn_fn): gate/up GEMVs, h = g/(1+exp(-g)) * u,
 * down GEMV over h. */
void orc_fused_ffn_silu(const float *x, size_t d, size_t d_ff, int type,
			const void *gate_w, const void *up_w, const void *down_w,
			int lanes, float *hidden, float *out)
{
	const int tg = ORC_QTYPE_GU(type), td = ORC_QTYPE_DN(type);
	/* Q8_DOT (nn.c:525-531, quant.c:656-668): K-quant gate/up rows take the
	 * integer dot against x quantized to Q8_K; every other type the fp32 dot */
	uint8_t *q8 = NULL;
	if ((tg == ORC_Q4_K || tg == ORC_Q6_K) && d % 256 == 0) {
		q8 = malloc(d / 256 * ORC_Q8K_BYTES);
		orc_quantize_row_q8K(x, q8, d);
	}
	for (size_t j = 0; j < d_ff; j++) {
		float g = q8 ? orc_dot_q8K(q8, gate_w, tg, j, d) : orc_dot_f32_quant(x, gate_w, tg, j, d, lanes);
		float u = q8 ? orc_dot_q8K(q8, up_w, tg, j, d) : orc_dot_f32_quant(x, up_w, tg, j, d, lanes);
		float sg = g / (1.0f + expf(-g));
		hidden[j] = sg * u;
	}
	free(q8);
	for (size_t j = 0; j < d; j++)
		out[j] = orc_dot_f32_quant(hidden, down_w, td, j, d_ff, lanes);
}

/* matmul.c:270-324 with a quantized rhs.  With k % 256 == 0 (the Q8_DOT
 * build) or m == 1 each element is one dot_f32_quant; otherwise rows are
 * dequantized and run through the fp32 lane-FMA tiles. */
void orc_gemm_q(const float *a, size_t m, size_t k, const void *b, int type,
		size_t n, int lanes, float *c)
{
	if (m == 1 || k % 256 == 0) {
		for (size_t i = 0; i < m; i++)
			for (size_t j = 0; j < n; j++)
				c[i * n + j] = 0.0f + orc_dot_f32_quant(a + i * k, b, type, j, k, lanes);
		return;
	}
	float *deq = malloc(k * sizeof(float));
	for (size_t j = 0; j < n; j++) {
		orc_dequant_row(b, type, j, deq, k);
		for (size_t i = 0; i < m; i++)
			c[i * n + j] = 0.0f + orc_dot_f32_f32(a + i * k, deq, k, lanes);
	}
	free(deq);
}

/* ------------------------------------------------------------------ */
/* MoE layer                                                            */
/* ------------------------------------------------------------------ */

/* olmoe.c:343-407 (renorm = 0) and llama.c:393-457 (renorm = 1) */
/* The per-(token, slot) terms y / (1 / w) of the combine (olmoe.c:397-404)
 * for the slots whose expert lies in [first, first + nlocal): z[t*K + s]
 * rows; the other rows are left as they are.  Adding the rows of a token in
 * slot order, starting from 0, gives orc_moe_ffn's output bit for bit —
 * the expert-parallel decomposition of the layer (each rank computes the
 * rows of its experts, the rows are exchanged, every rank combines). */
void orc_moe_slot_terms(const orc_moe_layer *L, const float *x, size_t T, size_t first,
			size_t nlocal, float *z, int32_t *ids_out, float *w_out)
{
	size_t d = L->d_model, NE = L->n_experts, K = L->top_k, F = L->d_ff;
	float *logits = malloc(T * NE * sizeof(float));
	float *hidden = malloc(F * sizeof(float));
	float *y = malloc(d * sizeof(float));
	int32_t ids[64];
	float w[64];

	orc_router_logits(x, T, d, L->router_w, NE, L->lanes, logits);
	if (L->router_bias)
		for (size_t t = 0; t < T; t++)
			for (size_t e = 0; e < NE; e++)
				logits[t * NE + e] = logits[t * NE + e] + L->router_bias[e];
	for (size_t t = 0; t < T; t++) {
		float *p = logits + t * NE;
		orc_softmax_1d(p, NE, L->lanes);
		orc_top_k(p, NE, ids, w, K, L->topk_mode);
		if (L->renorm) {
			float sum = 0.0f;
			for (size_t s = 0; s < K; s++)
				sum = sum + w[s];
			for (size_t s = 0; s < K; s++)
				w[s] = w[s] / sum;
		}
		for (size_t s = 0; s < K; s++) {
			size_t e = (size_t)ids[s];
			if (e < first || e >= first + nlocal)
				continue;
			const uint8_t *g = (const uint8_t *)L->gate + e * L->gate_stride;
			const uint8_t *u = (const uint8_t *)L->up + e * L->up_stride;
			const uint8_t *dn = (const uint8_t *)L->down + e * L->down_stride;
			orc_fused_ffn_silu(x + t * d, d, F, L->qtype, g, u, dn, L->lanes, hidden, y);
			float inv = 1.0f / w[s];
			float *zr = z + (t * K + s) * d;
			for (size_t j = 0; j < d; j++)
				zr[j] = y[j] / inv;
		}
		if (ids_out)
			memcpy(ids_out + t * K, ids, K * sizeof(int32_t));
		if (w_out)
			memcpy(w_out + t * K, w, K * sizeof(float));
	}
	free(logits);
	free(hidden);
	free(y);
}

void orc_moe_ffn(const orc_moe_layer *L, const float *x, size_t T, float *out,
		 int32_t *ids_out, float *w_out, float *probs_out)
{
	size_t d = L->d_model, NE = L->n_experts, K = L->top_k, F = L->d_ff;
	float *logits = malloc(T * NE * sizeof(float));
	float *hidden = malloc(F * sizeof(float));
	float *y = malloc(d * sizeof(float));
	int32_t ids[64];
	float w[64];

	memset(out, 0, T * d * sizeof(float));
	orc_router_logits(x, T, d, L->router_w, NE, L->lanes, logits);
	if (L->router_bias)
		for (size_t t = 0; t < T; t++)
			for (size_t e = 0; e < NE; e++)
				logits[t * NE + e] = logits[t * NE + e] + L->router_bias[e];

	for (size_t t = 0; t < T; t++) {
		float *p = logits + t * NE;
		orc_softmax_1d(p, NE, L->lanes);
		if (probs_out)
			memcpy(probs_out + t * NE, p, NE * sizeof(float));
		orc_top_k(p, NE, ids, w, K, L->topk_mode);
		if (L->renorm) {
			float sum = 0.0f;
			for (size_t s = 0; s < K; s++)
				sum = sum + w[s];
			for (size_t s = 0; s < K; s++)
				w[s] = w[s] / sum;
		}
		for (size_t s = 0; s < K; s++) {
			size_t e = (size_t)ids[s];
			const uint8_t *g = (const uint8_t *)L->gate + e * L->gate_stride;
			const uint8_t *u = (const uint8_t *)L->up + e * L->up_stride;
			const uint8_t *dn = (const uint8_t *)L->down + e * L->down_stride;
			orc_fused_ffn_silu(x + t * d, d, F, L->qtype, g, u, dn, L->lanes, hidden, y);
			/* tensor_div_scalar by 1/w, then tensor_add (olmoe.c:401-403) */
			float inv = 1.0f / w[s];
			float *o = out + t * d;
			for (size_t j = 0; j < d; j++)
				o[j] = o[j] + y[j] / inv;
		}
		if (ids_out)
			memcpy(ids_out + t * K, ids, K * sizeof(int32_t));
		if (w_out)
			memcpy(w_out + t * K, w, K * sizeof(float));
	}
	free(logits);
	free(hidden);
	free(y);
}
