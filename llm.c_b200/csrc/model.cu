// model.cu — the transformer around the MoE layers, on the device: token
// embedding, RMSNorm, QK-norm, RoPE, the KV cache, causal attention, the
// residual adds, lm_head and the greedy pick.  The OLMoE forward
// (models/olmoe/olmoe.c:409-502) and the llama/Mixtral forward
// (models/llama/llama.c:459-558) run as a sequence of launches on one
// stream; the decode step (T = 1) reads its token, position and cache size
// from a device state word, so it is captured once as a CUDA graph and
// replayed for every generated token.
//
// All arithmetic is fp32, as in the reference.  The cache keeps the
// reference's layout (kvcache.c:19-24: per layer [heads][context][head_len]
// fp32) in HBM.
#include "common.cuh"
#include "kernels.h"

#include <float.h>
#include <stdlib.h>

namespace moe {

namespace {

constexpr int kNormThreads = 256;

__device__ __forceinline__ float block_sum(float v, float *red)
{
	v = warp_sum(v);
	const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
	__syncthreads();   // red may still be read from a previous call
	if (lane == 0)
		red[warp] = v;
	__syncthreads();
	float t = 0.0f;
	if (threadIdx.x < 32) {
		t = threadIdx.x < (int)(blockDim.x / 32) ? red[threadIdx.x] : 0.0f;
		t = warp_sum(t);
		if (threadIdx.x == 0)
			red[0] = t;
	}
	__syncthreads();
	return red[0];
}

// element j of a GGUF row: dequant_row (quant.c:157-196): Q8_0 d * q,
// Q4_0 d * (nibble - 8) with element j < 16 in the low nibble of byte j
__device__ __forceinline__ float dequant_at(const uint8_t *row, int wtype, int j)
{
	if (wtype == 0)
		return reinterpret_cast<const float *>(row)[j];
	const int b = j / 32, k = j % 32;
	if (wtype == 1) {
		const uint8_t *blk = row + b * Q8_0_BYTES;
		const float d = __half2float(__ushort_as_half(
			(unsigned short)(blk[0] | (blk[1] << 8))));
		return d * (float)(int8_t)blk[2 + k];
	}
	const uint8_t *blk = row + b * Q4_0_BYTES;
	const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
	const int byte = blk[2 + (k & 15)];
	const int nib = k < 16 ? (byte & 15) : (byte >> 4);
	return d * (float)(nib - 8);
}

// rms_norm (nn.c:7-48): rms = sqrtf(sum(x^2) / n + 1e-5), out = (x / rms) * w
__device__ __forceinline__ void norm_row(const float *h, const float *w, float *out, int E,
					 float eps, float *red)
{
	float s = 0.0f;
	for (int j = threadIdx.x; j < E; j += blockDim.x)
		s = fmaf(h[j], h[j], s);
	const float sum = block_sum(s, red);
	const float rms = sqrtf(sum / (float)E + eps);
	for (int j = threadIdx.x; j < E; j += blockDim.x)
		out[j] = (h[j] / rms) * w[j];
}

// the rows of the tokens' ids (tensor_pick_rows, tensor.c:263-293) and
// their rms_norm; d_model <= 16 * 256 (REG): the row's loads all issued into
// registers first
template <bool REG>
__global__ void __launch_bounds__(kNormThreads)
embed_norm_kernel(const uint8_t *__restrict__ wte, int wtype, int64_t V, int E,
		  const int32_t *tok, const float *__restrict__ w, float eps,
		  float *__restrict__ hidden, float *__restrict__ out, int32_t *err)
{
	__shared__ float red[32];
	griddep_wait();
	griddep_launch_dependents();
	const int t = blockIdx.x;
	const int id = tok[t];
	float *h = hidden + (int64_t)t * E;
	const bool ok = id >= 0 && id < V;
	if (!ok && threadIdx.x == 0 && err)
		atomicOr(err, 1);
	const int64_t rb = wtype == 0 ? (int64_t)E * 4
			   : (int64_t)E / 32 * (wtype == 1 ? Q8_0_BYTES : Q4_0_BYTES);
	const uint8_t *row = wte + (ok ? (int64_t)id * rb : 0);
	if (REG) {
		float v[16];
#pragma unroll
		for (int k = 0; k < 16; k++) {
			const int j = threadIdx.x + k * kNormThreads;
			v[k] = (ok && j < E) ? dequant_at(row, wtype, j) : 0.0f;
		}
		float ss = 0.0f;
#pragma unroll
		for (int k = 0; k < 16; k++) {
			const int j = threadIdx.x + k * kNormThreads;
			if (j < E)
				h[j] = v[k];
			ss = fmaf(v[k], v[k], ss);
		}
		const float rms = sqrtf(block_sum(ss, red) / (float)E + eps);
#pragma unroll
		for (int k = 0; k < 16; k++) {
			const int j = threadIdx.x + k * kNormThreads;
			if (j < E)
				out[(int64_t)t * E + j] = (v[k] / rms) * w[j];
		}
	} else {
		for (int j = threadIdx.x; j < E; j += blockDim.x)
			h[j] = ok ? dequant_at(row, wtype, j) : 0.0f;
		__syncthreads();
		norm_row(h, w, out + (int64_t)t * E, E, eps, red);
	}
}

// tensor_add (tensor.c:334-353) then rms_norm.  d_model <= 16 * 256 and a
// multiple of 4 (VEC): four float4 per thread, every load issued before the
// first use (a strided loop would wait for each load in turn)
template <bool VEC>
__global__ void __launch_bounds__(kNormThreads)
add_norm_kernel(float *__restrict__ hidden, const float *__restrict__ delta,
		const float *__restrict__ w, int E, float eps, float *__restrict__ out)
{
	__shared__ float red[32];
	griddep_wait();
	griddep_launch_dependents();
	const int64_t o = (int64_t)blockIdx.x * E;
	float *h = hidden + o;
	if (VEC) {
		const int n4 = E / 4;
		float4 x[4], dl[4], wv[4];
#pragma unroll
		for (int k = 0; k < 4; k++) {
			const int i = threadIdx.x + k * kNormThreads;
			const bool in = i < n4;
			const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
			x[k] = in ? reinterpret_cast<const float4 *>(h)[i] : z;
			dl[k] = in && delta ? reinterpret_cast<const float4 *>(delta + o)[i] : z;
			wv[k] = in ? reinterpret_cast<const float4 *>(w)[i] : z;
		}
		float s = 0.0f;
#pragma unroll
		for (int k = 0; k < 4; k++) {
			x[k].x = __fadd_rn(x[k].x, dl[k].x);
			x[k].y = __fadd_rn(x[k].y, dl[k].y);
			x[k].z = __fadd_rn(x[k].z, dl[k].z);
			x[k].w = __fadd_rn(x[k].w, dl[k].w);
			s = fmaf(x[k].x, x[k].x, s);
			s = fmaf(x[k].y, x[k].y, s);
			s = fmaf(x[k].z, x[k].z, s);
			s = fmaf(x[k].w, x[k].w, s);
			const int i = threadIdx.x + k * kNormThreads;
			if (i < n4)
				reinterpret_cast<float4 *>(h)[i] = x[k];
		}
		const float rms = sqrtf(block_sum(s, red) / (float)E + eps);
#pragma unroll
		for (int k = 0; k < 4; k++) {
			const int i = threadIdx.x + k * kNormThreads;
			if (i < n4)
				reinterpret_cast<float4 *>(out + o)[i] =
					make_float4((x[k].x / rms) * wv[k].x, (x[k].y / rms) * wv[k].y,
						    (x[k].z / rms) * wv[k].z, (x[k].w / rms) * wv[k].w);
		}
	} else {
		for (int j = threadIdx.x; j < E; j += blockDim.x)
			h[j] = h[j] + (delta ? delta[o + j] : 0.0f);
		__syncthreads();
		norm_row(h, w, out + o, E, eps, red);
	}
}

// blockIdx.y: 0 = q, 1 = k, 2 = v of token blockIdx.x
__global__ void __launch_bounds__(kNormThreads) qk_rope_kernel(QkvArgs a)
{
	__shared__ float red[32];
	const int t = blockIdx.x, which = blockIdx.y;
	const int nq = a.H * a.HL, nk = a.KVH * a.HL;
	const float *src = a.qkv + (int64_t)t * (nq + 2 * nk) + (which == 0 ? 0 : which == 1 ? nq : nq + nk);
	const int n = which == 0 ? nq : nk;
	const int pos = a.pos[t];
	const int row = *a.size + t;
	if (pos < 0 || pos >= a.C || row < 0 || row >= a.C) {
		if (threadIdx.x == 0 && a.err)
			atomicOr(a.err, 2);
		return;
	}
	const float *nw = which == 0 ? a.q_norm : which == 1 ? a.k_norm : nullptr;
	float rms = 1.0f;
	if (nw) {
		float s = 0.0f;
		for (int j = threadIdx.x; j < n; j += blockDim.x)
			s = fmaf(src[j], src[j], s);
		rms = sqrtf(block_sum(s, red) / (float)n + a.eps);
	}
	const int half = a.HL / 2;
	const float2 *cs = a.rope + (int64_t)pos * half;
	for (int p = threadIdx.x; p < n / 2; p += blockDim.x) {
		float x0 = src[2 * p], x1 = src[2 * p + 1];
		int dst_h = (2 * p) / a.HL, e = (2 * p) % a.HL;
		if (which < 2) {
			if (nw) {
				x0 = (x0 / rms) * nw[2 * p];
				x1 = (x1 / rms) * nw[2 * p + 1];
			}
			// rope_apply (nn.c:192-219): consecutive pairs of each head
			const float2 c = cs[e / 2];
			const float y0 = x0 * c.x - x1 * c.y;
			const float y1 = x0 * c.y + x1 * c.x;
			x0 = y0;
			x1 = y1;
		}
		float *dst = which == 0 ? a.q_out + (int64_t)t * nq + 2 * p
			     : (which == 1 ? a.kc : a.vc) + ((int64_t)dst_h * a.C + row) * a.HL + e;
		dst[0] = x0;
		dst[1] = x1;
	}
}

// ---------------------------------------------------------------- attention
constexpr int kDecThreads = 128;   // 4 warps; head_len 128: 4 elements a lane

// decode: one query row per head, cache rows [c * 64, c * 64 + 64) of chunk
// c = blockIdx.y; partial (max, sum, o[HL]) to part[h][c]
__global__ void __launch_bounds__(kDecThreads)
attn_decode_kernel(const float *q, const float *kc, const float *vc, const int32_t *size, int H,
		   int KVH, int C, float scale_div, float *part)
{
	constexpr int HL = 128;
	__shared__ float4 so[4][32];
	__shared__ float sml[4][2];
	const int h = blockIdx.x, c = blockIdx.y, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
	const int AT = min(*size + 1, C);   // the host rotates a full cache first
	const int r0 = c * kAttnChunk, r1 = min(AT, r0 + kAttnChunk);
	float *pp = part + ((int64_t)h * gridDim.y + c) * (HL + 2);
	if (r0 >= r1)
		return;
	const int kvh = h / (H / KVH);
	const float4 qv = reinterpret_cast<const float4 *>(q + (int64_t)h * HL)[lane];
	const float *kb = kc + (int64_t)kvh * C * HL, *vb = vc + (int64_t)kvh * C * HL;
	float m = -FLT_MAX, l = 0.0f;
	float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
	for (int r = r0 + warp; r < r1; r += 4) {
		const float4 kv = reinterpret_cast<const float4 *>(kb + (int64_t)r * HL)[lane];
		const float4 vv = reinterpret_cast<const float4 *>(vb + (int64_t)r * HL)[lane];
		float s = qv.x * kv.x;
		s = fmaf(qv.y, kv.y, s);
		s = fmaf(qv.z, kv.z, s);
		s = fmaf(qv.w, kv.w, s);
		s = warp_sum(s) / scale_div;
		const float mn = fmaxf(m, s);
		const float f = expf(m - mn), p = expf(s - mn);
		l = fmaf(l, f, p);
		o.x = fmaf(o.x, f, p * vv.x);
		o.y = fmaf(o.y, f, p * vv.y);
		o.z = fmaf(o.z, f, p * vv.z);
		o.w = fmaf(o.w, f, p * vv.w);
		m = mn;
	}
	// merge the four warps (a warp without rows has l = 0)
	if (lane == 0) {
		sml[warp][0] = m;
		sml[warp][1] = l;
	}
	__syncthreads();
	float M = -FLT_MAX;
	for (int w = 0; w < 4; w++)
		if (sml[w][1] > 0.0f)
			M = fmaxf(M, sml[w][0]);
	const float fw = (l > 0.0f) ? expf(m - M) : 0.0f;
	so[warp][lane] = make_float4(o.x * fw, o.y * fw, o.z * fw, o.w * fw);
	__syncthreads();
	if (threadIdx.x < HL) {
		const float *sf = reinterpret_cast<const float *>(so);
		float acc = 0.0f;
		for (int w = 0; w < 4; w++)
			acc += sf[w * HL + threadIdx.x];
		pp[threadIdx.x] = acc;
	}
	if (threadIdx.x == 0) {
		float L = 0.0f;
		for (int w = 0; w < 4; w++)
			if (sml[w][1] > 0.0f)
				L = fmaf(sml[w][1], expf(sml[w][0] - M), L);
		pp[HL] = M;
		pp[HL + 1] = L;
	}
}

__global__ void __launch_bounds__(128)
attn_merge_kernel(const float *part, const int32_t *size, int C, int nsplit, float *out)
{
	constexpr int HL = 128;
	const int h = blockIdx.x, e = threadIdx.x;
	const int AT = max(1, min(*size + 1, C));
	const int ns = min(nsplit, (AT + kAttnChunk - 1) / kAttnChunk);
	const float *pp = part + (int64_t)h * nsplit * (HL + 2);
	float M = -FLT_MAX;
	for (int c = 0; c < ns; c++)
		M = fmaxf(M, pp[c * (HL + 2) + HL]);
	float L = 0.0f, acc = 0.0f;
	for (int c = 0; c < ns; c++) {
		const float f = expf(pp[c * (HL + 2) + HL] - M);
		L = fmaf(pp[c * (HL + 2) + HL + 1], f, L);
		acc = fmaf(pp[c * (HL + 2) + e], f, acc);
	}
	out[(int64_t)h * HL + e] = acc / L;
}

// Sum of squares of n floats (n % 4 == 0, n <= 16 * blockDim.x) with all
// loads issued before the first use: four float4 per thread
__device__ __forceinline__ float sumsq4(const float *__restrict__ v, int n, float *red)
{
	const int n4 = n / 4;
	float4 x[4];
#pragma unroll
	for (int k = 0; k < 4; k++) {
		const int i = threadIdx.x + k * blockDim.x;
		x[k] = i < n4 ? reinterpret_cast<const float4 *>(v)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
	}
	float s = 0.0f;
#pragma unroll
	for (int k = 0; k < 4; k++) {
		s = fmaf(x[k].x, x[k].x, s);
		s = fmaf(x[k].y, x[k].y, s);
		s = fmaf(x[k].z, x[k].z, s);
		s = fmaf(x[k].w, x[k].w, s);
	}
	return block_sum(s, red);
}

// One decode step (T = 1) of a layer's attention in one launch: grid (H,
// kStepSplits), 8 warps.  CTA c of head h takes cache rows
// [c AT / S, (c + 1) AT / S) of the AT = size + 1 rows.  Every CTA
// normalises (QK-norm over the whole vector, olmoe.c:455-459) and rotates
// (nn.c:192-219) its head's query; the CTA holding the new row (row `size`)
// does the same for its KV head's key, stores key and value into the cache
// and uses them from registers.  Each CTA's online-softmax partial goes to
// part[h][c]; the head's last CTA to finish (arrival counter cnt[h], reset by
// that CTA) merges them into out[h].  Each warp's first kStepU rows, the
// rope factors and the raw q (k, v) are loaded before the norm reductions,
// which would otherwise stand between dependent round trips; further rows
// go four at a time with their loads issued first.
constexpr int kStepThreads = 256, kStepWarps = kStepThreads / 32;
constexpr int kStepU = 8;   // cache rows per warp loaded before the norms

__global__ void __launch_bounds__(kStepThreads) attn_step_kernel(AttnStepArgs a)
{
	constexpr int HL = 128;
	__shared__ float4 so[kStepWarps][32];
	__shared__ float sml[kStepWarps][2];
	__shared__ float red[32];
	__shared__ int merge_here;
	griddep_wait();   // qkv comes from the projection launched before
	griddep_launch_dependents();
	const int h = blockIdx.x, c = blockIdx.y, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
	const int S = gridDim.y;
	const int size = *a.size, pos = *a.pos;
	if (size < 0 || size >= a.C || pos < 0 || pos >= a.C) {
		if (threadIdx.x == 0 && h == 0 && c == 0 && a.err)
			atomicOr(a.err, 2);
		return;
	}
	const int AT = size + 1;
	const int r0 = (int)((int64_t)c * AT / S), r1 = (int)((int64_t)(c + 1) * AT / S);
	const bool tail = c == S - 1;   // r1 == AT: this chunk holds the new row
	const int group = a.H / a.KVH, kvh = h / group;
	const int nq = a.H * HL, nk = a.KVH * HL;
	const float *qs = a.qkv, *ks = a.qkv + nq, *vs = a.qkv + nq + nk;
	const float *kb = a.kc + (int64_t)kvh * a.C * HL, *vb = a.vc + (int64_t)kvh * a.C * HL;
	const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
	// every load that does not wait for the norms goes out first: this
	// warp's first kStepU cache rows, the rope factors, the head's raw q (and
	// for the new row k, v) with their norm weights
	float4 kk[kStepU], vv[kStepU];
#pragma unroll
	for (int u = 0; u < kStepU; u++) {
		const int r = r0 + warp + u * kStepWarps;
		const bool in = r < r1 && r != size;
		kk[u] = in ? reinterpret_cast<const float4 *>(kb + (int64_t)r * HL)[lane] : z4;
		vv[u] = in ? reinterpret_cast<const float4 *>(vb + (int64_t)r * HL)[lane] : z4;
	}
	const float2 c0 = a.rope[(int64_t)pos * (HL / 2) + 2 * lane];
	const float2 c1 = a.rope[(int64_t)pos * (HL / 2) + 2 * lane + 1];
	const float4 qraw = reinterpret_cast<const float4 *>(qs + h * HL)[lane];
	const float4 qw = a.q_norm ? reinterpret_cast<const float4 *>(a.q_norm + h * HL)[lane] : z4;
	float4 kraw = z4, kw = z4, vnew = z4;
	if (tail) {
		kraw = reinterpret_cast<const float4 *>(ks + kvh * HL)[lane];
		kw = a.k_norm ? reinterpret_cast<const float4 *>(a.k_norm + kvh * HL)[lane] : z4;
		vnew = reinterpret_cast<const float4 *>(vs + kvh * HL)[lane];
	}
	float rq = 1.0f, rk = 1.0f;
	if (a.q_norm) {
		rq = sqrtf(sumsq4(qs, nq, red) / (float)nq + a.eps);
		if (tail)
			rk = sqrtf(sumsq4(ks, nk, red) / (float)nk + a.eps);
	}
	// lane owns elements 4 lane .. 4 lane + 3 of a head: pairs 2 lane, 2 lane + 1
	auto norm_rope = [&](float4 v, float4 w, bool norm, float r) {
		if (norm) {
			v.x = (v.x / r) * w.x;
			v.y = (v.y / r) * w.y;
			v.z = (v.z / r) * w.z;
			v.w = (v.w / r) * w.w;
		}
		return make_float4(v.x * c0.x - v.y * c0.y, v.x * c0.y + v.y * c0.x,
				   v.z * c1.x - v.w * c1.y, v.z * c1.y + v.w * c1.x);
	};
	const float4 qv = norm_rope(qraw, qw, a.q_norm != nullptr, rq);
	float4 knew = z4;
	if (tail) {
		knew = norm_rope(kraw, kw, a.k_norm != nullptr, rk);
		if (warp == 0 && h % group == 0) {
			reinterpret_cast<float4 *>(a.kc + ((int64_t)kvh * a.C + size) * HL)[lane] = knew;
			reinterpret_cast<float4 *>(a.vc + ((int64_t)kvh * a.C + size) * HL)[lane] = vnew;
		}
	}
	float m = -FLT_MAX, l = 0.0f;
	float4 o = z4;
	auto take = [&](float4 k4, float4 v4) {
		float s = qv.x * k4.x;
		s = fmaf(qv.y, k4.y, s);
		s = fmaf(qv.z, k4.z, s);
		s = fmaf(qv.w, k4.w, s);
		s = warp_sum(s) / a.scale_div;
		const float mn = fmaxf(m, s);
		const float f = expf(m - mn), p = expf(s - mn);
		l = fmaf(l, f, p);
		o.x = fmaf(o.x, f, p * v4.x);
		o.y = fmaf(o.y, f, p * v4.y);
		o.z = fmaf(o.z, f, p * v4.z);
		o.w = fmaf(o.w, f, p * v4.w);
		m = mn;
	};
#pragma unroll
	for (int u = 0; u < kStepU; u++) {
		const int r = r0 + warp + u * kStepWarps;
		if (r < r1)
			take(r == size ? knew : kk[u], r == size ? vnew : vv[u]);
	}
	// rows past the first batch (long caches): four at a time, loads first
	for (int rb = r0 + warp + kStepU * kStepWarps; rb < r1; rb += kStepWarps * 4) {
		float4 k4[4], v4[4];
#pragma unroll
		for (int u = 0; u < 4; u++) {
			const int r = rb + u * kStepWarps;
			const bool in = r < r1 && r != size;
			k4[u] = in ? reinterpret_cast<const float4 *>(kb + (int64_t)r * HL)[lane] : z4;
			v4[u] = in ? reinterpret_cast<const float4 *>(vb + (int64_t)r * HL)[lane] : z4;
		}
#pragma unroll
		for (int u = 0; u < 4; u++) {
			const int r = rb + u * kStepWarps;
			if (r < r1)
				take(r == size ? knew : k4[u], r == size ? vnew : v4[u]);
		}
	}
	if (lane == 0) {
		sml[warp][0] = m;
		sml[warp][1] = l;
	}
	__syncthreads();
	float M = -FLT_MAX;
	for (int w = 0; w < kStepWarps; w++)
		if (sml[w][1] > 0.0f)
			M = fmaxf(M, sml[w][0]);
	const float fw = (l > 0.0f) ? expf(m - M) : 0.0f;
	so[warp][lane] = make_float4(o.x * fw, o.y * fw, o.z * fw, o.w * fw);
	__syncthreads();
	float *pp = a.part + ((int64_t)h * S + c) * (HL + 2);
	if (threadIdx.x < HL) {
		const float *sf = reinterpret_cast<const float *>(so);
		float acc = 0.0f;
		for (int w = 0; w < kStepWarps; w++)
			acc += sf[w * HL + threadIdx.x];
		pp[threadIdx.x] = acc;
	}
	if (threadIdx.x == 0) {
		float L = 0.0f;
		for (int w = 0; w < kStepWarps; w++)
			if (sml[w][1] > 0.0f)
				L = fmaf(sml[w][1], expf(sml[w][0] - M), L);
		pp[HL] = M;
		pp[HL + 1] = L;   // 0 for a CTA without rows
	}
	// the head's last CTA merges (release: partial, then the count)
	__threadfence();
	__syncthreads();
	if (threadIdx.x == 0)
		merge_here = atomicAdd(a.cnt + h, 1) == S - 1;
	__syncthreads();
	if (!merge_here)
		return;
	__threadfence();
	const float *hp = a.part + (int64_t)h * S * (HL + 2);
	// every partial's loads first (S <= 16), then the merge
	float Mq[16], Lq[16], Oq[16];
#pragma unroll
	for (int q = 0; q < 16; q++) {
		const bool in = q < S;
		Mq[q] = in ? __ldcg(hp + q * (HL + 2) + HL) : -FLT_MAX;
		Lq[q] = in ? __ldcg(hp + q * (HL + 2) + HL + 1) : 0.0f;
		Oq[q] = in && threadIdx.x < HL ? __ldcg(hp + q * (HL + 2) + threadIdx.x) : 0.0f;
	}
	float Mx = -FLT_MAX;
#pragma unroll
	for (int q = 0; q < 16; q++)
		if (Lq[q] > 0.0f)
			Mx = fmaxf(Mx, Mq[q]);
	float Ls = 0.0f, acc = 0.0f;
#pragma unroll
	for (int q = 0; q < 16; q++)
		if (Lq[q] > 0.0f) {
			const float f = expf(Mq[q] - Mx);
			Ls = fmaf(Lq[q], f, Ls);
			acc = fmaf(Oq[q], f, acc);
		}
	if (threadIdx.x < HL)
		a.out[(int64_t)h * HL + threadIdx.x] = acc / Ls;
	if (threadIdx.x == 0)
		a.cnt[h] = 0;   // ready for the next launch
}

// prefill: 16 query rows of one head per CTA against 64-row tiles of the
// cache, online softmax (the reference forms the full masked score matrix,
// olmoe.c:300-312: scores / sqrt(head_len), -1e4 above the diagonal, which
// exp() turns into exact zeros, softmax_2d; the same sums in another order)
constexpr int kPfRows = 16, kPfKeys = 64, kPfThreads = 256, kPfStride = 132;
constexpr size_t kPfSmem =
	(size_t)(kPfRows * kPfStride + kPfKeys * kPfStride + kPfKeys * 128 + kPfRows * kPfKeys) * 4;

__global__ void __launch_bounds__(kPfThreads)
attn_prefill_kernel(const float *q, const float *kc, const float *vc, const int32_t *size, int T,
		    int H, int KVH, int C, float scale_div, float *out)
{
	constexpr int HL = 128;
	extern __shared__ float4 smem_f4[];
	float *Qs = reinterpret_cast<float *>(smem_f4);
	float *Ks = Qs + kPfRows * kPfStride;
	float *Vs = Ks + kPfKeys * kPfStride;
	float *Ps = Vs + kPfKeys * HL;
	const int h = blockIdx.x, t0 = blockIdx.y * kPfRows, tid = threadIdx.x;
	const int r = tid / 16, cc = tid % 16;
	const int base = *size;
	const int nq = H * HL;
	const int kvh = h / (H / KVH);
	const float *kb = kc + (int64_t)kvh * C * HL, *vb = vc + (int64_t)kvh * C * HL;
	for (int i = tid; i < kPfRows * 32; i += kPfThreads) {
		const int rr = i / 32, e4 = i % 32;
		const float4 v = t0 + rr < T ? reinterpret_cast<const float4 *>(
						      q + (int64_t)(t0 + rr) * nq + (int64_t)h * HL)[e4]
					     : make_float4(0.f, 0.f, 0.f, 0.f);
		*reinterpret_cast<float4 *>(Qs + rr * kPfStride + 4 * e4) = v;
	}
	const int t = t0 + r;
	// last cache row any row here sees (the host keeps size + T <= C)
	const int last = min(base + min(t0 + kPfRows, T) - 1, C - 1);
	const int lim = base + t;                            // this row sees rows <= lim
	float m = -FLT_MAX, l = 0.0f;
	float4 o0 = make_float4(0.f, 0.f, 0.f, 0.f), o1 = o0;
	for (int k0 = 0; k0 <= last; k0 += kPfKeys) {
		__syncthreads();   // the previous tile's Ks/Vs/Ps are consumed
		for (int i = tid; i < kPfKeys * 32; i += kPfThreads) {
			const int rr = i / 32, e4 = i % 32;
			const bool in = k0 + rr <= last;
			const float4 kv = in ? reinterpret_cast<const float4 *>(kb + (int64_t)(k0 + rr) * HL)[e4]
					     : make_float4(0.f, 0.f, 0.f, 0.f);
			const float4 vv = in ? reinterpret_cast<const float4 *>(vb + (int64_t)(k0 + rr) * HL)[e4]
					     : make_float4(0.f, 0.f, 0.f, 0.f);
			*reinterpret_cast<float4 *>(Ks + rr * kPfStride + 4 * e4) = kv;
			*reinterpret_cast<float4 *>(Vs + rr * HL + 4 * e4) = vv;
		}
		__syncthreads();
		float s[4];
		const float *qr = Qs + r * kPfStride;
#pragma unroll
		for (int i = 0; i < 4; i++) {
			const float *kr = Ks + (cc + 16 * i) * kPfStride;
			float acc = 0.0f;
#pragma unroll 8
			for (int e = 0; e < HL; e += 4) {
				const float4 a = *reinterpret_cast<const float4 *>(qr + e);
				const float4 b = *reinterpret_cast<const float4 *>(kr + e);
				acc = fmaf(a.x, b.x, acc);
				acc = fmaf(a.y, b.y, acc);
				acc = fmaf(a.z, b.z, acc);
				acc = fmaf(a.w, b.w, acc);
			}
			s[i] = (k0 + cc + 16 * i <= lim) ? acc / scale_div : -FLT_MAX;
		}
		float mx = fmaxf(fmaxf(s[0], s[1]), fmaxf(s[2], s[3]));
#pragma unroll
		for (int off = 8; off; off >>= 1)
			mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
		const float mn = fmaxf(m, mx);
		const float f = expf(m - mn);
		float ps = 0.0f;
#pragma unroll
		for (int i = 0; i < 4; i++) {
			const float p = s[i] == -FLT_MAX ? 0.0f : expf(s[i] - mn);
			Ps[r * kPfKeys + cc + 16 * i] = p;
			ps += p;
		}
#pragma unroll
		for (int off = 8; off; off >>= 1)
			ps += __shfl_xor_sync(0xffffffffu, ps, off);
		l = fmaf(l, f, ps);
		m = mn;
		o0.x *= f; o0.y *= f; o0.z *= f; o0.w *= f;
		o1.x *= f; o1.y *= f; o1.z *= f; o1.w *= f;
		__syncthreads();
		const int nk = min(kPfKeys, last + 1 - k0);
		for (int j = 0; j < nk; j++) {
			const float p = Ps[r * kPfKeys + j];
			const float4 v0 = *reinterpret_cast<const float4 *>(Vs + j * HL + 4 * cc);
			const float4 v1 = *reinterpret_cast<const float4 *>(Vs + j * HL + 64 + 4 * cc);
			o0.x = fmaf(p, v0.x, o0.x); o0.y = fmaf(p, v0.y, o0.y);
			o0.z = fmaf(p, v0.z, o0.z); o0.w = fmaf(p, v0.w, o0.w);
			o1.x = fmaf(p, v1.x, o1.x); o1.y = fmaf(p, v1.y, o1.y);
			o1.z = fmaf(p, v1.z, o1.z); o1.w = fmaf(p, v1.w, o1.w);
		}
	}
	if (t < T) {
		float *dst = out + (int64_t)t * nq + (int64_t)h * HL;
		const float il = 1.0f / l;
		*reinterpret_cast<float4 *>(dst + 4 * cc) =
			make_float4(o0.x * il, o0.y * il, o0.z * il, o0.w * il);
		*reinterpret_cast<float4 *>(dst + 64 + 4 * cc) =
			make_float4(o1.x * il, o1.y * il, o1.z * il, o1.w * il);
	}
}

// ---------------------------------------------------------------- decode state
// state = {tok, pos, size, model_pos}: the pick of this step becomes the next
// step's token; olmoe_decode (olmoe.c:510-520): the cache grows by one row,
// positions past the context are replaced by the cache size
constexpr int kArgCtas = 64, kArgThreads = 256;

__device__ __forceinline__ bool pick_better(float v, int i, float w, int j)
{
	// the first maximum: a larger value, or the same value at a lower index
	return j >= 0 && (i < 0 || w > v || (w == v && j < i));
}

__device__ __forceinline__ void block_argmax(float &best, int &idx, float *bv, int *bi)
{
	for (int off = 16; off; off >>= 1) {
		const float w = __shfl_xor_sync(0xffffffffu, best, off);
		const int j = __shfl_xor_sync(0xffffffffu, idx, off);
		if (pick_better(best, idx, w, j)) {
			best = w;
			idx = j;
		}
	}
	const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
	if (lane == 0) {
		bv[warp] = best;
		bi[warp] = idx;
	}
	__syncthreads();
	if (warp == 0) {
		best = lane < (int)(blockDim.x / 32) ? bv[lane] : -FLT_MAX;
		idx = lane < (int)(blockDim.x / 32) ? bi[lane] : -1;
		for (int off = 16; off; off >>= 1) {
			const float w = __shfl_xor_sync(0xffffffffu, best, off);
			const int j = __shfl_xor_sync(0xffffffffu, idx, off);
			if (pick_better(best, idx, w, j)) {
				best = w;
				idx = j;
			}
		}
	}
}

// kArgCtas CTAs take contiguous slices of the logits (four loads per
// thread in flight); the last CTA to finish (counter cnt, reset by it)
// reduces their partial maxima in slice order and updates the state
__global__ void __launch_bounds__(kArgThreads)
argmax_advance_kernel(const float *logits, int V, int C, int32_t *state, int32_t *picks,
		      int pick_cap, int advance, float *pv, int32_t *pi, int32_t *cnt)
{
	__shared__ float bv[32];
	__shared__ int bi[32];
	__shared__ int last;
	griddep_wait();
	const int chunk = (V + gridDim.x - 1) / gridDim.x;
	const int b0 = blockIdx.x * chunk, b1 = min(V, b0 + chunk);
	float best = -FLT_MAX;
	int idx = -1;
	for (int i0 = b0 + threadIdx.x; i0 < b1; i0 += 4 * kArgThreads) {
		float v[4];
#pragma unroll
		for (int u = 0; u < 4; u++) {
			const int i = i0 + u * kArgThreads;
			v[u] = i < b1 ? logits[i] : -FLT_MAX;
		}
#pragma unroll
		for (int u = 0; u < 4; u++) {
			const int i = i0 + u * kArgThreads;
			if (i < b1 && (idx < 0 || v[u] > best)) {
				best = v[u];
				idx = i;
			}
		}
	}
	block_argmax(best, idx, bv, bi);
	if (threadIdx.x == 0) {
		pv[blockIdx.x] = best;
		pi[blockIdx.x] = idx;
		__threadfence();
		last = atomicAdd(cnt, 1) == (int)gridDim.x - 1;
	}
	__syncthreads();
	if (!last)
		return;
	__threadfence();
	best = -FLT_MAX;
	idx = -1;
	for (int c = threadIdx.x; c < (int)gridDim.x; c += blockDim.x) {
		const float w = __ldcg(pv + c);
		const int j = __ldcg(pi + c);
		if (pick_better(best, idx, w, j)) {
			best = w;
			idx = j;
		}
	}
	__syncthreads();
	block_argmax(best, idx, bv, bi);
	if (threadIdx.x == 0) {
		*cnt = 0;
		const int tok = idx < 0 ? 0 : idx;
		state[0] = tok;
		picks[state[6] % pick_cap] = tok;
		state[6] += 1;
		if (advance) {
			const int size = state[2] + 1, mpos = state[3] + 1;
			state[2] = size;
			state[3] = mpos;
			state[1] = mpos >= C ? size : mpos;
		}
	}
}

// one pass of the cache rotation (kvcache.c:29-55): rows [drop + p*drop ..)
// -> [p*drop ..), which never overlap within a pass
__global__ void kv_shift_kernel(float *kc, float *vc, int C, int HL, int from, int to, int rows)
{
	const int64_t per = (int64_t)rows * HL;
	const int64_t head = blockIdx.y;            // (layer, kv head) of K then V
	float *base = (blockIdx.z ? vc : kc) + head * C * HL;
	for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < per;
	     i += (int64_t)gridDim.x * blockDim.x)
		base[(int64_t)to * HL + i] = base[(int64_t)from * HL + i];
}

template <typename... P, typename... A>
cudaError_t launch_k(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
		     bool pdl, A... args)
{
	cudaLaunchConfig_t cfg{};
	cfg.gridDim = grid;
	cfg.blockDim = block;
	cfg.dynamicSmemBytes = smem;
	cfg.stream = st;
	cudaLaunchAttribute at[1];
	at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	at[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = at;
	cfg.numAttrs = pdl ? 1 : 0;
	return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace

cudaError_t launch_embed_norm(const void *wte, int wtype, int64_t V, int E, const int32_t *tok,
			      int T, const float *w, float eps, float *hidden, float *out,
			      int32_t *err, cudaStream_t st, bool pdl)
{
	if (T <= 0)
		return cudaSuccess;
	if (E <= 16 * kNormThreads)
		return launch_k(embed_norm_kernel<true>, dim3(T), dim3(kNormThreads), 0, st, pdl,
				static_cast<const uint8_t *>(wte), wtype, V, E, tok, w, eps, hidden, out,
				err);
	return launch_k(embed_norm_kernel<false>, dim3(T), dim3(kNormThreads), 0, st, pdl,
			static_cast<const uint8_t *>(wte), wtype, V, E, tok, w, eps, hidden, out, err);
}

cudaError_t launch_add_norm(float *hidden, const float *delta, const float *w, int T, int E,
			    float eps, float *out, cudaStream_t st, bool pdl)
{
	if (T <= 0)
		return cudaSuccess;
	if (E % 4 == 0 && E <= 16 * kNormThreads)
		return launch_k(add_norm_kernel<true>, dim3(T), dim3(kNormThreads), 0, st, pdl, hidden,
				delta, w, E, eps, out);
	return launch_k(add_norm_kernel<false>, dim3(T), dim3(kNormThreads), 0, st, pdl, hidden,
			delta, w, E, eps, out);
}

cudaError_t launch_qk_rope(const QkvArgs &a, cudaStream_t st)
{
	if (a.T <= 0)
		return cudaSuccess;
	if (a.HL % 2 || a.KVH <= 0 || a.H % a.KVH)
		return cudaErrorInvalidValue;
	qk_rope_kernel<<<dim3(a.T, 3), kNormThreads, 0, st>>>(a);
	return cudaGetLastError();
}

cudaError_t launch_attention(const float *q, const float *kc, const float *vc, const int32_t *size,
			     int T, int H, int KVH, int HL, int C, float scale_div, float *part,
			     float *out, cudaStream_t st)
{
	if (T <= 0)
		return cudaSuccess;
	if (HL != 128 || KVH <= 0 || H % KVH)
		return cudaErrorInvalidValue;
	if (T == 1) {
		const int ns = attn_splits(C);
		attn_decode_kernel<<<dim3(H, ns), kDecThreads, 0, st>>>(q, kc, vc, size, H, KVH, C,
									 scale_div, part);
		if (cudaError_t e = cudaGetLastError())
			return e;
		attn_merge_kernel<<<H, 128, 0, st>>>(part, size, C, ns, out);
		return cudaGetLastError();
	}
	static bool attr = false;
	if (!attr) {
		if (cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel,
							 cudaFuncAttributeMaxDynamicSharedMemorySize,
							 (int)kPfSmem))
			return e;
		attr = true;
	}
	attn_prefill_kernel<<<dim3(H, (T + kPfRows - 1) / kPfRows), kPfThreads, kPfSmem, st>>>(
		q, kc, vc, size, T, H, KVH, C, scale_div, out);
	return cudaGetLastError();
}

bool pdl_enabled()
{
	static const bool on = [] {
		const char *e = getenv("MOE_PDL");
		return !(e && e[0] == '0');
	}();
	return on;
}

cudaError_t launch_attn_step(const AttnStepArgs &a, cudaStream_t st)
{
	if (a.KVH <= 0 || a.H % a.KVH)
		return cudaErrorInvalidValue;
	if (a.H * 128 > 16 * kStepThreads || a.KVH * 128 > 16 * kStepThreads)
		return cudaErrorInvalidValue;   // sumsq4's reach
	cudaLaunchConfig_t cfg{};
	cfg.gridDim = dim3(a.H, attn_step_splits(a.C));
	cfg.blockDim = dim3(kStepThreads);
	cfg.dynamicSmemBytes = 0;
	cfg.stream = st;
	cudaLaunchAttribute at[1];
	at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	at[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = at;
	cfg.numAttrs = pdl_enabled() ? 1 : 0;
	return cudaLaunchKernelEx(&cfg, attn_step_kernel, a);
}

cudaError_t launch_argmax_advance(const float *logits, int V, int C, int32_t *state,
				  int32_t *picks, int pick_cap, int advance, float *scratch,
				  cudaStream_t st, bool pdl)
{
	// scratch: kArgCtas floats, kArgCtas ints, one counter (zero)
	float *pv = scratch;
	int32_t *pi = reinterpret_cast<int32_t *>(scratch + kArgCtas);
	int32_t *cnt = pi + kArgCtas;
	return launch_k(argmax_advance_kernel, dim3(kArgCtas), dim3(kArgThreads), 0, st, pdl, logits,
			V, C, state, picks, pick_cap, advance, pv, pi, cnt);
}

cudaError_t launch_kv_shift(float *kc, float *vc, int L, int KVH, int C, int HL, int keep,
			    int drop, cudaStream_t st)
{
	if (keep <= 0 || drop <= 0)
		return cudaSuccess;
	for (int done = 0; done < keep; done += drop) {
		const int rows = min(drop, keep - done);
		kv_shift_kernel<<<dim3(16, L * KVH, 2), 256, 0, st>>>(kc, vc, C, HL, drop + done, done,
								       rows);
		if (cudaError_t e = cudaGetLastError())
			return e;
	}
	return cudaSuccess;
}

}  // namespace moe

// ====================================================================== engine
#include "moe_b200.h"

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <utility>
#include <vector>

namespace {

int mfail(int code, const char *fmt, ...)
{
	char buf[512];
	va_list ap;
	va_start(ap, fmt);
	vsnprintf(buf, sizeof buf, fmt, ap);
	va_end(ap);
	moe::set_last_error(buf);
	return code;
}

int mcuda(cudaError_t e, const char *what)
{
	return mfail(e == cudaErrorMemoryAllocation ? MOE_ERR_NOMEM : MOE_ERR_CUDA, "%s: %s", what,
		     cudaGetErrorString(e));
}

#define MCK(call)                                                  \
	do {                                                       \
		cudaError_t e_ = (call);                           \
		if (e_ != cudaSuccess)                             \
			return mcuda(e_, #call);                   \
	} while (0)

#define MRC(call)                                                  \
	do {                                                       \
		int rc_ = (call);                                  \
		if (rc_ != MOE_OK)                                 \
			return rc_;                                \
	} while (0)

int64_t row_bytes_of(int type, int64_t cols)
{
	return type == MOE_F32 ? cols * 4 : cols / 32 * (type == MOE_Q8_0 ? Q8_0_BYTES : Q4_0_BYTES);
}

// device state words
// S_ERR: bits 1 (token id) and 2 (position / cache row) of this file's
// kernels; S_PERR: the projections' bounded waits; S_STEP: picks made
enum { S_TOK = 0, S_POS = 1, S_SIZE = 2, S_MPOS = 3, S_ERR = 4, S_PERR = 5, S_STEP = 6, S_WORDS = 8 };

}  // namespace

struct moe_model {
	moe_model_desc d{};
	int64_t L = 0, E = 0, H = 0, KVH = 0, HL = 0, V = 0, C = 0, NE = 0, K = 0, F = 0;
	int64_t nq = 0, nk = 0;          // H*HL, KVH*HL
	float scale_div = 1.0f;          // sqrt(head_len) (olmoe.c:158)
	bool qk_norm = false, renorm = false;
	cudaStream_t st = nullptr;
	std::vector<void *> owned;       // every device allocation
	size_t bytes = 0;
	// weights
	const void *wte = nullptr;
	int wte_t = 0;
	const void *lm = nullptr;
	int lm_t = 0;
	const float *out_norm = nullptr;
	struct Layer {
		const float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr,
			    *k_norm = nullptr;
		const void *wqkv = nullptr, *wo = nullptr;
		int qkv_t = 0, o_t = 0;
		moe_layer *moe = nullptr;                // MoE FFN
		const void *wg = nullptr, *wu = nullptr, *wd = nullptr;  // dense FFN
		int ffn_t = 0;
	};
	std::vector<Layer> layers;
	float2 *rope = nullptr;          // [C][HL/2]
	float *kc = nullptr, *vc = nullptr;  // [L][KVH][C][HL]
	// activations (capacity cap rows)
	int64_t cap = 0;
	float *hidden = nullptr, *xn = nullptr, *qkv = nullptr, *q = nullptr, *att = nullptr,
	      *proj = nullptr, *ffn = nullptr, *gate = nullptr, *up = nullptr;
	float *hidden2 = nullptr;        // the decode step's second residual buffer
	int32_t *attn_cnt = nullptr;     // [H] arrival counters of the fused attention
	bool fused_step = false;         // T = 1 through the fused kernels
	int32_t *tok = nullptr, *pos = nullptr;
	std::vector<void *> act;         // the activation buffers (regrown)
	float *part = nullptr;           // decode attention partials
	float *logits = nullptr;         // [V]
	int32_t *state = nullptr;        // device S_WORDS
	int32_t *hstate = nullptr;       // pinned mirror
	int32_t *picks = nullptr;        // greedy picks, ring of pick_cap
	float *argbuf = nullptr;         // the pick's partial maxima and counter
	int64_t pick_cap = 0;
	int64_t logits_row = -1;         // row of xn whose logits m->logits holds
	int64_t size = 0, mpos = 0;      // host mirrors of the cache size and model position
	int64_t last_T = 0;              // rows of the last forward's output
	moe::DenseScratch ds;
	cudaGraph_t graph = nullptr;
	cudaGraphExec_t gexec = nullptr;
	bool graphable = true;
	std::vector<int64_t> graph_rows;  // each MoE layer's scratch rows at capture
	cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};  // generate: start, first pick, end
	bool timed = false;
};

namespace {

int dalloc(moe_model *m, void **p, size_t bytes)
{
	*p = nullptr;
	if (!bytes)
		return MOE_OK;
	MCK(cudaMalloc(p, bytes));
	m->owned.push_back(*p);
	m->bytes += bytes;
	return MOE_OK;
}

const void *host_ptr(const moe_tensor_t *t)
{
	return t->type == MOE_F32 ? (const void *)t->data : t->qdata;
}

// copy a GGUF view into HBM after checking its element count (gguf.c
// checks the same) and type
int upload(moe_model *m, const moe_tensor_t *t, int64_t rows, int64_t cols, bool f32_only,
	   const char *what, const void **dev, int *type)
{
	if (!t || !host_ptr(t))
		return mfail(MOE_ERR_INVALID, "moe_model_create: %s missing", what);
	if (t->type != MOE_F32 && t->type != MOE_Q8_0 && t->type != MOE_Q4_0)
		return mfail(MOE_ERR_UNSUPPORTED, "moe_model_create: %s has dtype %d", what, t->type);
	if (f32_only && t->type != MOE_F32)
		return mfail(MOE_ERR_UNSUPPORTED, "moe_model_create: %s must be F32", what);
	if ((int64_t)t->totlen != rows * cols || (t->type != MOE_F32 && cols % 32))
		return mfail(MOE_ERR_INVALID, "moe_model_create: %s has %llu elements, expected "
			     "%lld x %lld", what, (unsigned long long)t->totlen, (long long)rows,
			     (long long)cols);
	const size_t bytes = (size_t)(rows * row_bytes_of(t->type, cols));
	void *p;
	MRC(dalloc(m, &p, bytes));
	MCK(cudaMemcpy(p, host_ptr(t), bytes, cudaMemcpyDefault));   // host or device views
	*dev = p;
	if (type)
		*type = t->type;
	return MOE_OK;
}

// rope_apply's angles (nn.c:201-206) with the host's libm, the library the
// reference calls: freq_i = 1 / theta^(2i / HL), angle = pos * freq_i
int build_rope(moe_model *m)
{
	const int64_t half = m->HL / 2;
	std::vector<float2> tab((size_t)(m->C * half));
	for (int64_t i = 0; i < half; i++) {
		const float freq = 1.0f / powf(m->d.rope_theta, (float)(2 * i) / (float)m->HL);
		for (int64_t p = 0; p < m->C; p++) {
			const float angle = (float)p * freq;
			tab[(size_t)(p * half + i)] = make_float2(cosf(angle), sinf(angle));
		}
	}
	void *p;
	MRC(dalloc(m, &p, tab.size() * sizeof(float2)));
	MCK(cudaMemcpy(p, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice));
	m->rope = static_cast<float2 *>(p);
	return MOE_OK;
}

int ensure_act(moe_model *m, int64_t T)
{
	if (T <= m->cap)
		return MOE_OK;
	MCK(cudaStreamSynchronize(m->st));
	for (void *p : m->act)
		cudaFree(p);
	m->act.clear();
	m->cap = 0;
	const int64_t E = m->E, nqkv = m->nq + 2 * m->nk;
	const int64_t ffw = m->NE ? 0 : m->F;
	auto get = [&](auto **p, size_t bytes) -> int {
		void *v = nullptr;
		MCK(cudaMalloc(&v, bytes));
		m->act.push_back(v);
		*p = static_cast<std::remove_reference_t<decltype(**p)> *>(v);
		return MOE_OK;
	};
	MRC(get(&m->hidden, T * E * 4));
	MRC(get(&m->hidden2, T * E * 4));
	MRC(get(&m->xn, T * E * 4));
	MRC(get(&m->qkv, T * nqkv * 4));
	MRC(get(&m->q, T * m->nq * 4));
	MRC(get(&m->att, T * m->nq * 4));
	MRC(get(&m->proj, T * E * 4));
	MRC(get(&m->ffn, T * E * 4));
	if (ffw) {
		MRC(get(&m->gate, T * ffw * 4));
		MRC(get(&m->up, T * ffw * 4));
	}
	MRC(get(&m->tok, T * 4));
	MRC(get(&m->pos, T * 4));
	m->cap = T;
	return MOE_OK;
}

}  // namespace

namespace {

// The decode step (T = 1) through the fused kernels, each launched as a
// programmatic dependent of the one before: per layer the QKV GEMV takes the
// residual add and attn_norm into its prologue (the residual stream moves
// between two buffers), one launch does QK-norm + RoPE + cache row +
// attention, then the O GEMV, the add + ffn_norm, and the MoE layer.
int forward_step(moe_model *m, const int32_t *tok_d, const int32_t *pos_d)
{
	const int E = (int)m->E;
	const float eps = 1e-5f;
	const bool pdl = moe::pdl_enabled();
	int32_t *size_d = m->state + S_SIZE, *err = m->state + S_ERR, *perr = m->state + S_PERR;
	MCK(moe::launch_embed_norm(m->wte, m->wte_t, m->V, E, tok_d, 1, m->layers[0].attn_norm, eps,
				   m->hidden, m->xn, err, m->st, pdl));
	const int64_t nqkv = m->nq + 2 * m->nk;
	const size_t per_layer = (size_t)(m->KVH * m->C * m->HL);
	float *R = m->hidden, *R2 = m->hidden2;
	const float *D = nullptr;
	for (int64_t l = 0; l < m->L; l++) {
		const moe_model::Layer &ly = m->layers[l];
		moe::NormIn nin;
		nin.hidden = R;
		nin.delta = D;
		nin.weight = ly.attn_norm;
		nin.hidden_out = R2;
		nin.eps = eps;
		MCK(moe::launch_gemv_norm(ly.wqkv, ly.qkv_t, nqkv, E, nin, m->qkv, perr, pdl, m->st));
		std::swap(R, R2);
		moe::AttnStepArgs a{};
		a.qkv = m->qkv;
		a.q_norm = ly.q_norm;
		a.k_norm = ly.k_norm;
		a.rope = m->rope;
		a.pos = pos_d;
		a.size = size_d;
		a.kc = m->kc + l * per_layer;
		a.vc = m->vc + l * per_layer;
		a.part = m->part;
		a.cnt = m->attn_cnt;
		a.out = m->att;
		a.H = (int)m->H;
		a.KVH = (int)m->KVH;
		a.C = (int)m->C;
		a.eps = eps;
		a.scale_div = m->scale_div;
		a.err = err;
		MCK(moe::launch_attn_step(a, m->st));
		MCK(moe::launch_gemv1(ly.wo, ly.o_t, E, m->nq, m->att, m->proj, perr, m->st, pdl));
		MCK(moe::launch_add_norm(R, m->proj, ly.ffn_norm, 1, E, eps, m->xn, m->st, pdl));
		MRC(moe_layer_forward(ly.moe, m->xn, m->ffn, 1, m->renorm ? MOE_RENORM : 0, m->st));
		D = m->ffn;
	}
	MCK(moe::launch_add_norm(R, D, m->out_norm, 1, E, eps, m->xn, m->st, pdl));
	return MOE_OK;
}

// One forward over T tokens (olmoe.c:409-502 / llama.c:459-558) on m->st:
// tok_d/pos_d are device arrays of T ids and positions, the cache grows
// from state[S_SIZE].  Leaves the final-normed rows in m->xn.
int forward(moe_model *m, int64_t T, const int32_t *tok_d, const int32_t *pos_d)
{
	if (T == 1 && m->fused_step)
		return forward_step(m, tok_d, pos_d);
	const int E = (int)m->E;
	const float eps = 1e-5f;
	int32_t *size_d = m->state + S_SIZE, *err = m->state + S_ERR, *perr = m->state + S_PERR;
	MCK(moe::launch_embed_norm(m->wte, m->wte_t, m->V, E, tok_d, (int)T, m->layers[0].attn_norm,
				   eps, m->hidden, m->xn, err, m->st));
	const int64_t nqkv = m->nq + 2 * m->nk;
	const size_t per_layer = (size_t)(m->KVH * m->C * m->HL);
	for (int64_t l = 0; l < m->L; l++) {
		const moe_model::Layer &ly = m->layers[l];
		MRC(moe::dense_forward(m->ds, ly.wqkv, ly.qkv_t, nqkv, E, m->xn, T, m->qkv, perr, m->st));
		moe::QkvArgs a{};
		a.qkv = m->qkv;
		a.q_norm = ly.q_norm;
		a.k_norm = ly.k_norm;
		a.rope = m->rope;
		a.pos = pos_d;
		a.size = size_d;
		a.q_out = m->q;
		a.kc = m->kc + l * per_layer;
		a.vc = m->vc + l * per_layer;
		a.T = (int)T;
		a.H = (int)m->H;
		a.KVH = (int)m->KVH;
		a.HL = (int)m->HL;
		a.C = (int)m->C;
		a.eps = eps;
		a.err = err;
		MCK(moe::launch_qk_rope(a, m->st));
		MCK(moe::launch_attention(m->q, a.kc, a.vc, size_d, (int)T, (int)m->H, (int)m->KVH,
					  (int)m->HL, (int)m->C, m->scale_div, m->part, m->att, m->st));
		MRC(moe::dense_forward(m->ds, ly.wo, ly.o_t, E, m->nq, m->att, T, m->proj, perr, m->st));
		MCK(moe::launch_add_norm(m->hidden, m->proj, ly.ffn_norm, (int)T, E, eps, m->xn, m->st));
		MRC(moe_layer_forward(ly.moe, m->xn, m->ffn, T, m->renorm ? MOE_RENORM : 0, m->st));
		const float *next = l + 1 < m->L ? m->layers[l + 1].attn_norm : m->out_norm;
		MCK(moe::launch_add_norm(m->hidden, m->ffn, next, (int)T, E, eps, m->xn, m->st));
	}
	return MOE_OK;
}

// the host's cache size and position into the device state (S_POS, S_SIZE,
// S_MPOS; S_TOK too when tok >= 0)
int write_state(moe_model *m, int64_t pos, int tok)
{
	m->hstate[S_TOK] = tok;
	m->hstate[S_POS] = (int32_t)pos;
	m->hstate[S_SIZE] = (int32_t)m->size;
	m->hstate[S_MPOS] = (int32_t)m->mpos;
	if (tok >= 0)
		MCK(cudaMemcpyAsync(m->state, m->hstate, 4 * sizeof(int32_t), cudaMemcpyHostToDevice,
				    m->st));
	else
		MCK(cudaMemcpyAsync(m->state + S_POS, m->hstate + S_POS, 3 * sizeof(int32_t),
				    cudaMemcpyHostToDevice, m->st));
	// the pinned words may be rewritten by the next call before this copy ran
	MCK(cudaStreamSynchronize(m->st));
	return MOE_OK;
}

// kvcache_rotate (kvcache.c:29-55): keep the newest context/2 rows
int rotate(moe_model *m)
{
	const int64_t keep = std::min<int64_t>(m->C / 2, m->size);
	const int64_t drop = m->size - keep;
	MCK(moe::launch_kv_shift(m->kc, m->vc, (int)m->L, (int)m->KVH, (int)m->C, (int)m->HL,
				 (int)keep, (int)drop, m->st));
	m->size = keep;
	return MOE_OK;
}

// the decode step on the state's token: forward, lm_head, pick, advance
int decode_step_body(moe_model *m)
{
	MRC(forward(m, 1, m->state + S_TOK, m->state + S_POS));
	const bool pdl = m->fused_step && moe::pdl_enabled();
	if (m->fused_step)
		MCK(moe::launch_gemv1(m->lm, m->lm_t, m->V, m->E, m->xn, m->logits, m->state + S_PERR,
				      m->st, pdl));
	else
		MRC(moe::dense_forward(m->ds, m->lm, m->lm_t, m->V, m->E, m->xn, 1, m->logits,
				       m->state + S_PERR, m->st));
	MCK(moe::launch_argmax_advance(m->logits, (int)m->V, (int)m->C, m->state, m->picks,
				       (int)m->pick_cap, 1, m->argbuf, m->st, pdl));
	return MOE_OK;
}

void drop_graph(moe_model *m)
{
	if (m->gexec)
		cudaGraphExecDestroy(m->gexec);
	if (m->graph)
		cudaGraphDestroy(m->graph);
	m->gexec = nullptr;
	m->graph = nullptr;
}

int capture(moe_model *m)
{
	// a MoE layer whose scratch grew (a larger prefill) moved the buffers
	// the graph holds: capture again
	if (m->gexec) {
		bool same = m->graph_rows.size() == m->layers.size();
		for (size_t i = 0; same && i < m->layers.size(); i++)
			same = moe::layer_scratch_rows(m->layers[i].moe) == m->graph_rows[i];
		if (same)
			return MOE_OK;
		drop_graph(m);
	}
	MCK(cudaStreamSynchronize(m->st));
	MCK(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
	const int rc = decode_step_body(m);
	cudaGraph_t g = nullptr;
	cudaError_t e = cudaStreamEndCapture(m->st, &g);
	if (rc != MOE_OK) {
		if (g)
			cudaGraphDestroy(g);
		return rc;
	}
	if (e == cudaSuccess) {
		m->graph = g;
		e = cudaGraphInstantiate(&m->gexec, g, 0);
	}
	if (e != cudaSuccess) {
		// a step that cannot be captured runs eagerly (same launches)
		cudaGetLastError();
		drop_graph(m);
		m->graphable = false;
		return MOE_OK;
	}
	m->graph_rows.clear();
	for (const auto &ly : m->layers)
		m->graph_rows.push_back(moe::layer_scratch_rows(ly.moe));
	return MOE_OK;
}

int take_state_error(moe_model *m)
{
	MCK(cudaStreamSynchronize(m->st));
	int32_t e[2] = {0, 0};
	MCK(cudaMemcpy(e, m->state + S_ERR, 8, cudaMemcpyDeviceToHost));
	if (e[0] || e[1]) {
		MCK(cudaMemset(m->state + S_ERR, 0, 8));
		if (e[1])
			return mfail(MOE_ERR_TIMEOUT, "moe_model: a bounded wait expired in a projection");
		return mfail(MOE_ERR_INVALID, "moe_model: %s%s", (e[0] & 1) ? "token id outside the "
			     "vocabulary; " : "", (e[0] & 2) ? "position or cache row out of range" : "");
	}
	for (const auto &ly : m->layers)
		if (ly.moe)
			MRC(moe_layer_status(ly.moe));
	return MOE_OK;
}

}  // namespace

// ====================================================================== C ABI
namespace {

int create_layers(moe_model *m)
{
	const moe_model_desc &d = m->d;
	const int64_t E = m->E, F = m->F, NE = m->NE;
	m->layers.resize((size_t)m->L);
	for (int64_t l = 0; l < m->L; l++) {
		moe_model::Layer &ly = m->layers[l];
		char what[64];
		const void *p;
		snprintf(what, sizeof what, "blk.%lld.attn_norm", (long long)l);
		MRC(upload(m, d.attn_norm[l], 1, E, true, what, &p, nullptr));
		ly.attn_norm = static_cast<const float *>(p);
		snprintf(what, sizeof what, "blk.%lld.ffn_norm", (long long)l);
		MRC(upload(m, d.ffn_norm[l], 1, E, true, what, &p, nullptr));
		ly.ffn_norm = static_cast<const float *>(p);
		if (m->qk_norm) {
			snprintf(what, sizeof what, "blk.%lld.attn_q_norm", (long long)l);
			MRC(upload(m, d.attn_q_norm[l], 1, m->nq, true, what, &p, nullptr));
			ly.q_norm = static_cast<const float *>(p);
			snprintf(what, sizeof what, "blk.%lld.attn_k_norm", (long long)l);
			MRC(upload(m, d.attn_k_norm[l], 1, m->nk, true, what, &p, nullptr));
			ly.k_norm = static_cast<const float *>(p);
		}
		// q, k, v as one [nq + 2 nk, E] matrix: one projection launch
		const moe_tensor_t *qkv[3] = {d.attn_q[l], d.attn_k[l], d.attn_v[l]};
		const int64_t rows[3] = {m->nq, m->nk, m->nk};
		int t0 = -1;
		for (int i = 0; i < 3; i++) {
			if (!qkv[i] || !host_ptr(qkv[i]))
				return mfail(MOE_ERR_INVALID, "moe_model_create: blk.%lld q/k/v missing",
					     (long long)l);
			if (t0 < 0)
				t0 = qkv[i]->type;
			if (qkv[i]->type != t0 || (t0 != MOE_Q8_0 && t0 != MOE_Q4_0))
				return mfail(MOE_ERR_UNSUPPORTED, "moe_model_create: blk.%lld q/k/v must "
					     "share one Q8_0/Q4_0 type", (long long)l);
			if ((int64_t)qkv[i]->totlen != rows[i] * E)
				return mfail(MOE_ERR_INVALID, "moe_model_create: blk.%lld q/k/v element "
					     "count", (long long)l);
		}
		const int64_t rb = row_bytes_of(t0, E);
		void *w;
		MRC(dalloc(m, &w, (size_t)((m->nq + 2 * m->nk) * rb)));
		int64_t off = 0;
		for (int i = 0; i < 3; i++) {
			MCK(cudaMemcpy(static_cast<uint8_t *>(w) + off, host_ptr(qkv[i]),
				       (size_t)(rows[i] * rb), cudaMemcpyDefault));
			off += rows[i] * rb;
		}
		ly.wqkv = w;
		ly.qkv_t = t0;
		snprintf(what, sizeof what, "blk.%lld.attn_output", (long long)l);
		MRC(upload(m, d.attn_output[l], E, m->nq, false, what, &ly.wo, &ly.o_t));
		if (ly.o_t == MOE_F32)
			return mfail(MOE_ERR_UNSUPPORTED, "moe_model_create: %s must be Q8_0/Q4_0", what);
		// the FFN: this library's MoE layer (a dense FFN is one expert that
		// every token takes with weight 1: softmax of one logit is 1.0 and
		// y / (1 / 1.0) = y)
		const int64_t ne = NE ? NE : 1, k = NE ? m->K : 1;
		const float *router = nullptr;
		if (NE) {
			snprintf(what, sizeof what, "blk.%lld.ffn_gate_inp", (long long)l);
			MRC(upload(m, d.ffn_gate_inp[l], NE, E, true, what, &p, nullptr));
			router = static_cast<const float *>(p);
		} else {
			void *z;
			MRC(dalloc(m, &z, (size_t)E * 4));
			MCK(cudaMemset(z, 0, (size_t)E * 4));
			router = static_cast<const float *>(z);
		}
		std::vector<const void *> g((size_t)ne), u((size_t)ne), dn((size_t)ne);
		int qt = -1;
		auto expert_mats = [&](const moe_tensor_t *const *arr, int64_t r, int64_t c,
				       const char *nm, std::vector<const void *> &ptr) -> int {
			if (d.arch == MOE_ARCH_OLMOE) {
				// one 3-D tensor [NE, r, c]: expert e at e * r * row_bytes
				const moe_tensor_t *t = arr[l];
				const void *base;
				int tt;
				char w2[64];
				snprintf(w2, sizeof w2, "blk.%lld.%s_exps", (long long)l, nm);
				MRC(upload(m, t, NE * r, c, false, w2, &base, &tt));
				if (qt >= 0 && tt != qt)
					return mfail(MOE_ERR_UNSUPPORTED, "moe_model_create: mixed expert "
						     "types");
				qt = tt;
				for (int64_t e = 0; e < NE; e++)
					ptr[(size_t)e] = static_cast<const uint8_t *>(base) +
							 e * r * row_bytes_of(tt, c);
			} else {
				for (int64_t e = 0; e < ne; e++) {
					const moe_tensor_t *t = arr[l * ne + e];
					int tt;
					char w2[64];
					snprintf(w2, sizeof w2, "blk.%lld.%s.%lld", (long long)l, nm,
						 (long long)e);
					MRC(upload(m, t, r, c, false, w2, &ptr[(size_t)e], &tt));
					if (qt >= 0 && tt != qt)
						return mfail(MOE_ERR_UNSUPPORTED, "moe_model_create: mixed "
							     "expert types");
					qt = tt;
				}
			}
			return MOE_OK;
		};
		MRC(expert_mats(d.ffn_gate, F, E, "ffn_gate", g));
		MRC(expert_mats(d.ffn_up, F, E, "ffn_up", u));
		MRC(expert_mats(d.ffn_down, E, F, "ffn_down", dn));
		if (qt != MOE_Q8_0 && qt != MOE_Q4_0)
			return mfail(MOE_ERR_UNSUPPORTED, "moe_model_create: experts must be Q8_0/Q4_0");
		moe_layer_desc ld{};
		ld.d_model = E;
		ld.d_ff = F;
		ld.n_experts = ne;
		ld.top_k = k;
		ld.qtype = qt;
		ld.flags = 0;
		ld.router_w = router;
		ld.router_bias = nullptr;
		ld.gate = g.data();
		ld.up = u.data();
		ld.down = dn.data();
		MRC(moe_layer_create(&ly.moe, &ld));
		ly.ffn_t = qt;
	}
	return MOE_OK;
}

void free_model(moe_model *m)
{
	if (!m)
		return;
	if (m->st)
		cudaStreamSynchronize(m->st);
	drop_graph(m);
	for (auto &ly : m->layers)
		if (ly.moe)
			moe_layer_destroy(ly.moe);
	for (void *p : m->act)
		cudaFree(p);
	for (void *p : m->owned)
		cudaFree(p);
	if (m->hstate)
		cudaFreeHost(m->hstate);
	for (cudaEvent_t e : m->ev)
		if (e)
			cudaEventDestroy(e);
	moe::dense_scratch_free(m->ds);
	delete m;
}

int prefill_impl(moe_model *m, const int *tok, const int *pos, int64_t T)
{
	if (T <= 0)
		return MOE_OK;
	if (m->size + T > m->C)
		return mfail(MOE_ERR_INVALID, "moe_model_prefill: %lld cached + %lld new rows exceed "
			     "the context %lld", (long long)m->size, (long long)T, (long long)m->C);
	for (int64_t t = 0; t < T; t++)
		if (pos[t] < 0 || pos[t] >= m->C || tok[t] < 0 || tok[t] >= m->V)
			return mfail(MOE_ERR_INVALID, "moe_model_prefill: token %lld: id %d / position "
				     "%d out of range", (long long)t, tok[t], pos[t]);
	if (T > m->cap)
		drop_graph(m);   // the graph holds the activation pointers
	MRC(ensure_act(m, T));
	MRC(write_state(m, 0, -1));
	MCK(cudaMemcpyAsync(m->tok, tok, (size_t)T * 4, cudaMemcpyHostToDevice, m->st));
	MCK(cudaMemcpyAsync(m->pos, pos, (size_t)T * 4, cudaMemcpyHostToDevice, m->st));
	MRC(forward(m, T, m->tok, m->pos));
	m->size += T;
	m->last_T = T;
	m->logits_row = -1;
	return MOE_OK;
}

// one decode step of token tok at position pos (olmoe_decode, olmoe.c:510-520)
// (host_tok: tok comes from the caller; otherwise the device state holds the
// previous pick, and its position and cache size, which the last step's
// pick advanced, are rewritten only when sync_state is set or the cache
// rotated)
int decode_impl(moe_model *m, int tok, int64_t pos, bool host_tok, bool sync_state)
{
	bool rotated = false;
	if (m->size >= m->C) {
		MRC(rotate(m));
		rotated = true;
	}
	if (pos >= m->C)
		pos = m->size;
	if (host_tok && (tok < 0 || tok >= m->V))
		return mfail(MOE_ERR_INVALID, "moe_model_decode: token id %d", tok);
	if (pos < 0)
		return mfail(MOE_ERR_INVALID, "moe_model_decode: position %lld", (long long)pos);
	MRC(ensure_act(m, 1));
	if (host_tok || sync_state || rotated)
		MRC(write_state(m, pos, host_tok ? tok : -1));
	if (m->graphable)
		MRC(capture(m));
	if (m->gexec)
		MCK(cudaGraphLaunch(m->gexec, m->st));
	else
		MRC(decode_step_body(m));
	m->size += 1;
	m->mpos += 1;
	m->last_T = 1;
	m->logits_row = 0;
	return MOE_OK;
}

}  // namespace

extern "C" {

int moe_model_create(moe_model **out, const moe_model_desc *desc)
{
	if (!out || !desc)
		return mfail(MOE_ERR_INVALID, "moe_model_create: null argument");
	*out = nullptr;
	MRC(moe::ensure_library());
	const moe_model_desc &d = *desc;
	if (d.arch != MOE_ARCH_OLMOE && d.arch != MOE_ARCH_LLAMA)
		return mfail(MOE_ERR_INVALID, "moe_model_create: arch %d", d.arch);
	const int64_t kvh = d.n_kv_heads ? d.n_kv_heads : d.n_heads;
	if (d.n_layers <= 0 || d.d_model <= 0 || d.d_model % 32 || d.n_heads <= 0 || kvh <= 0 ||
	    d.n_heads % kvh || d.head_len != 128 || d.vocab <= 0 || d.context <= 0 ||
	    d.context > (1 << 20) || d.n_experts < 0 || d.n_experts > 256 || d.d_ff <= 0 ||
	    d.d_ff % 32 || (d.n_experts && (d.top_k <= 0 || d.top_k > d.n_experts)))
		return mfail(MOE_ERR_INVALID, "moe_model_create: shape (layers %lld d %lld heads "
			     "%lld/%lld head_len %lld vocab %lld context %lld experts %lld top %lld "
			     "d_ff %lld; head_len must be 128)", (long long)d.n_layers,
			     (long long)d.d_model, (long long)d.n_heads, (long long)kvh,
			     (long long)d.head_len, (long long)d.vocab, (long long)d.context,
			     (long long)d.n_experts, (long long)d.top_k, (long long)d.d_ff);
	if (d.arch == MOE_ARCH_OLMOE && (kvh != d.n_heads || d.n_heads * d.head_len != d.d_model ||
					 !d.n_experts || !d.attn_q_norm || !d.attn_k_norm))
		return mfail(MOE_ERR_INVALID, "moe_model_create: OLMoE needs heads x head_len = "
			     "d_model, experts and QK-norm weights (olmoe.c:155)");
	if (!d.token_embd || !d.output || !d.output_norm || !d.attn_norm || !d.attn_q ||
	    !d.attn_k || !d.attn_v || !d.attn_output || !d.ffn_norm || !d.ffn_gate || !d.ffn_up ||
	    !d.ffn_down || (d.n_experts && !d.ffn_gate_inp))
		return mfail(MOE_ERR_INVALID, "moe_model_create: missing tensor arrays");
	moe_model *m = new moe_model();
	m->d = d;
	m->L = d.n_layers;
	m->E = d.d_model;
	m->H = d.n_heads;
	m->KVH = kvh;
	m->HL = d.head_len;
	m->V = d.vocab;
	m->C = d.context;
	m->NE = d.n_experts;
	m->K = d.top_k;
	m->F = d.d_ff;
	m->nq = m->H * m->HL;
	m->nk = m->KVH * m->HL;
	m->scale_div = sqrtf((float)m->HL);
	m->qk_norm = d.arch == MOE_ARCH_OLMOE;
	m->renorm = d.arch == MOE_ARCH_LLAMA && d.n_experts > 0;
	m->st = moe::library_stream();
	int rc = MOE_OK;
	auto step = [&](int r) {
		if (rc == MOE_OK)
			rc = r;
		return rc == MOE_OK;
	};
	const void *p;
	if (step(upload(m, d.token_embd, m->V, m->E, false, "token_embd", &m->wte, &m->wte_t)) &&
	    step(upload(m, d.output, m->V, m->E, false, "output", &m->lm, &m->lm_t)) &&
	    step(m->lm_t == MOE_F32 ? mfail(MOE_ERR_UNSUPPORTED, "moe_model_create: output must "
					    "be Q8_0/Q4_0") : MOE_OK) &&
	    step(upload(m, d.output_norm, 1, m->E, true, "output_norm", &p, nullptr))) {
		m->out_norm = static_cast<const float *>(p);
		step(create_layers(m));
	}
	void *v;
	const size_t cache = (size_t)(m->L * m->KVH * m->C * m->HL) * 4;
	if (rc == MOE_OK && step(dalloc(m, &v, cache)))
		m->kc = static_cast<float *>(v);
	if (rc == MOE_OK && step(dalloc(m, &v, cache)))
		m->vc = static_cast<float *>(v);
	if (rc == MOE_OK && step(build_rope(m)) &&
	    step(dalloc(m, &v, (size_t)(m->H * std::max(moe::attn_splits((int)m->C),
						       moe::attn_step_splits((int)m->C)) *
					(m->HL + 2)) * 4)))
		m->part = static_cast<float *>(v);
	if (rc == MOE_OK && step(dalloc(m, &v, (size_t)m->V * 4)))
		m->logits = static_cast<float *>(v);
	m->pick_cap = 4096;
	if (rc == MOE_OK && step(dalloc(m, &v, (size_t)m->pick_cap * 4)))
		m->picks = static_cast<int32_t *>(v);
	if (rc == MOE_OK && step(dalloc(m, &v, 4096))) {
		m->argbuf = static_cast<float *>(v);
		const cudaError_t e = cudaMemset(v, 0, 4096);
		if (e != cudaSuccess)
			step(mcuda(e, "moe_model_create: pick scratch"));
	}
	if (rc == MOE_OK && step(dalloc(m, &v, S_WORDS * 4))) {
		m->state = static_cast<int32_t *>(v);
		cudaError_t e = cudaMemset(v, 0, S_WORDS * 4);
		if (e == cudaSuccess)
			e = cudaMallocHost(&m->hstate, S_WORDS * 4);
		if (e != cudaSuccess)
			step(mcuda(e, "moe_model_create: state"));
	}
	if (rc != MOE_OK) {
		free_model(m);
		return rc;
	}
	// the decode step goes into a CUDA graph when every projection of one
	// row is the single-row GEMV (no host copy inside the step)
	const uintptr_t al = 256;
	m->graphable = moe::gemv1_supported(m->lm_t, m->V, m->E, (uintptr_t)m->lm, al, al);
	for (const auto &ly : m->layers)
		m->graphable = m->graphable &&
			       moe::gemv1_supported(ly.qkv_t, m->nq + 2 * m->nk, m->E,
						    (uintptr_t)ly.wqkv, al, al) &&
			       moe::gemv1_supported(ly.o_t, m->E, m->nq, (uintptr_t)ly.wo, al, al);
	// the fused decode step: tensor-core GEMVs for every one-row projection
	// (the QKV one with the norm in its prologue)
	m->fused_step = m->graphable && moe::gemv_norm_supported(m->lm_t, m->E, (uintptr_t)m->lm);
	for (const auto &ly : m->layers)
		m->fused_step = m->fused_step &&
				moe::gemv_norm_supported(ly.qkv_t, m->E, (uintptr_t)ly.wqkv) &&
				moe::gemv_norm_supported(ly.o_t, m->nq, (uintptr_t)ly.wo);
	if (m->fused_step) {
		void *c = nullptr;
		rc = dalloc(m, &c, (size_t)m->H * 4);
		if (rc == MOE_OK) {
			const cudaError_t e = cudaMemset(c, 0, (size_t)m->H * 4);
			if (e != cudaSuccess)
				rc = mcuda(e, "moe_model_create: counters");
		}
		m->attn_cnt = static_cast<int32_t *>(c);
		if (rc != MOE_OK) {
			free_model(m);
			return rc;
		}
	}
	// one eager decode step on token 0 into the empty cache: every layer's
	// one-row scratch and every kernel attribute exist before a capture
	rc = ensure_act(m, 1);
	if (rc == MOE_OK)
		rc = write_state(m, 0, 0);
	if (rc == MOE_OK)
		rc = decode_step_body(m);
	if (rc == MOE_OK) {
		const cudaError_t e = cudaStreamSynchronize(m->st);
		rc = e == cudaSuccess ? take_state_error(m) : mcuda(e, "moe_model_create: warm-up");
	}
	if (rc == MOE_OK) {
		const cudaError_t e = cudaMemset(m->state, 0, S_WORDS * 4);
		if (e != cudaSuccess)
			rc = mcuda(e, "moe_model_create: state");
	}
	if (rc != MOE_OK) {
		free_model(m);
		return rc;
	}
	*out = m;
	return MOE_OK;
}

int moe_model_destroy(moe_model *m)
{
	free_model(m);
	return MOE_OK;
}

int moe_model_reset(moe_model *m)
{
	if (!m)
		return mfail(MOE_ERR_INVALID, "moe_model_reset: null model");
	m->size = 0;
	m->mpos = 0;
	m->last_T = 0;
	m->logits_row = -1;
	return MOE_OK;
}

int moe_model_prefill(moe_model *m, const int *tok, const int *pos, size_t T, float *output)
{
	if (!m || (T && (!tok || !pos)))
		return mfail(MOE_ERR_INVALID, "moe_model_prefill: null argument");
	MRC(prefill_impl(m, tok, pos, (int64_t)T));
	if (output && T)
		MCK(cudaMemcpyAsync(output, m->xn, T * m->E * 4, cudaMemcpyDeviceToHost, m->st));
	return take_state_error(m);
}

int moe_model_decode(moe_model *m, int tok, int pos, float *output)
{
	if (!m)
		return mfail(MOE_ERR_INVALID, "moe_model_decode: null model");
	MRC(decode_impl(m, tok, pos, true, true));
	if (output)
		MCK(cudaMemcpyAsync(output, m->xn, m->E * 4, cudaMemcpyDeviceToHost, m->st));
	return take_state_error(m);
}

int moe_model_logits(moe_model *m, size_t row, float *logits)
{
	if (!m || !logits)
		return mfail(MOE_ERR_INVALID, "moe_model_logits: null argument");
	if ((int64_t)row >= m->last_T)
		return mfail(MOE_ERR_INVALID, "moe_model_logits: row %zu of %lld", row,
			     (long long)m->last_T);
	if (m->logits_row != (int64_t)row) {
		MRC(moe::dense_forward(m->ds, m->lm, m->lm_t, m->V, m->E, m->xn + row * m->E, 1,
				       m->logits, m->state + S_PERR, m->st));
		m->logits_row = (int64_t)row;
	}
	MCK(cudaMemcpyAsync(logits, m->logits, m->V * 4, cudaMemcpyDeviceToHost, m->st));
	return take_state_error(m);
}

int moe_model_generate(moe_model *m, const int *prompt, size_t T, int n, int eos, int *tokens)
{
	if (!m || (T && !prompt) || n < 0 || !tokens)
		return mfail(MOE_ERR_INVALID, "moe_model_generate: bad argument");
	if (T == 0)
		return mfail(MOE_ERR_INVALID, "moe_model_generate: empty prompt");
	std::vector<int> pos(T);
	for (size_t i = 0; i < T; i++)
		pos[i] = (int)(m->mpos + (int64_t)i);
	for (cudaEvent_t &e : m->ev)
		if (!e)
			MCK(cudaEventCreate(&e));
	m->timed = false;
	MCK(cudaEventRecord(m->ev[0], m->st));
	MRC(prefill_impl(m, prompt, pos.data(), (int64_t)T));
	m->mpos += (int64_t)T;
	// the first pick, from the last prompt row (olmoe.c:559-564)
	MRC(moe::dense_forward(m->ds, m->lm, m->lm_t, m->V, m->E, m->xn + (T - 1) * m->E, 1,
			       m->logits, m->state + S_PERR, m->st));
	MCK(cudaMemsetAsync(m->state + S_STEP, 0, 4, m->st));
	MCK(moe::launch_argmax_advance(m->logits, (int)m->V, (int)m->C, m->state, m->picks,
				       (int)m->pick_cap, 0, m->argbuf, m->st));
	MCK(cudaEventRecord(m->ev[1], m->st));
	int made = 1;
	int last = -1;
	auto read_picks = [&](int from, int to) -> int {
		// picks [from, to) out of the ring (to - from <= pick_cap)
		for (int i = from; i < to;) {
			const int slot = (int)(i % m->pick_cap);
			const int cnt = std::min<int>(to - i, (int)(m->pick_cap - slot));
			MCK(cudaMemcpyAsync(tokens + i, m->picks + slot, (size_t)cnt * 4,
					    cudaMemcpyDeviceToHost, m->st));
			i += cnt;
		}
		MCK(cudaStreamSynchronize(m->st));
		return MOE_OK;
	};
	int copied = 0;
	while (made <= n) {
		if (eos >= 0) {
			MRC(read_picks(copied, made));
			copied = made;
			last = tokens[made - 1];
			if (last == eos)
				break;
		} else if (made - copied >= m->pick_cap) {
			MRC(read_picks(copied, made));
			copied = made;
		}
		// olmoe_decode: rotate a full cache; positions past the context
		// become the cache size
		const int64_t p = m->mpos;
		MRC(decode_impl(m, 0, p, false, made == 1));
		made++;
	}
	MCK(cudaEventRecord(m->ev[2], m->st));
	if (copied < made)
		MRC(read_picks(copied, made));
	MRC(take_state_error(m));
	m->timed = true;
	return made;
}

int moe_model_timing(moe_model *m, float *prefill_ms, float *decode_ms)
{
	if (!m || !m->timed)
		return mfail(MOE_ERR_INVALID, "moe_model_timing: no completed moe_model_generate");
	MCK(cudaEventSynchronize(m->ev[2]));
	if (prefill_ms)
		MCK(cudaEventElapsedTime(prefill_ms, m->ev[0], m->ev[1]));
	if (decode_ms)
		MCK(cudaEventElapsedTime(decode_ms, m->ev[1], m->ev[2]));
	return MOE_OK;
}

int moe_model_status(moe_model *m)
{
	if (!m)
		return mfail(MOE_ERR_INVALID, "moe_model_status: null model");
	return take_state_error(m);
}

int moe_model_mode(moe_model *m)
{
	if (!m)
		return mfail(MOE_ERR_INVALID, "moe_model_mode: null model");
	return (m->gexec ? 1 : 0) | (m->fused_step ? 2 : 0) |
	       (m->fused_step && moe::pdl_enabled() ? 4 : 0);
}

int moe_model_info(moe_model *m, int64_t *cache_size, int64_t *pos, size_t *device_bytes)
{
	if (!m)
		return mfail(MOE_ERR_INVALID, "moe_model_info: null model");
	if (cache_size)
		*cache_size = m->size;
	if (pos)
		*pos = m->mpos;
	if (device_bytes)
		*device_bytes = m->bytes;
	return MOE_OK;
}

}  // extern "C"
