// router.cu — K1: router logits, softmax + top-k, and the expert dispatch.
//
// The router reproduces the reference's floating-point operation order so
// that expert ids match the CPU path bit for bit:
//   * logits: matmul.c:91-131 / :169-245 keep one fp32 FMA chain per SIMD
//     lane (lane j sums elements j, j+L, j+2L, ... in order) and reduce the
//     L lanes with a halving tree; L = 16 for the AVX-512 build, 8 for AVX2.
//     Here each chain is one thread of an L-thread group.
//   * softmax: nn.c:221-262 — max, exp(l - max) stored, lane-wise sums of
//     the exps reduced by the same tree, sequential tail, then division.
//   * top-k: nn.c:276-308, whose insertion scheme seeds all k slots with
//     element 0.  Its result equals: rank the sequence [p0 (k copies), p1,
//     p2, ...] by (value desc, position asc), keep ranks < k, output slot
//     k-1-rank.  Each element's rank is computed independently here.
#include "common.cuh"
#include "kernels.h"
#include "route_core.cuh"

namespace moe {

// ---------------------------------------------------------------------
// logits[t, e] = 0 + dot(x[t, :], w[e, :]) with LANES-lane FMA chains.
// Block: 256 threads = 256/LANES groups.  Tile: 8 tokens x 8 experts; each
// group owns one token and EPG experts of the tile.
// ---------------------------------------------------------------------
constexpr int kRouterTT = 8;
constexpr int kRouterET = 8;

template <int LANES>
__global__ void __launch_bounds__(256)
router_logits_kernel(const float *__restrict__ x, const float *__restrict__ w,
		     float *__restrict__ logits, int T, int d, int NE)
{
	extern __shared__ float xs[];  // [kRouterTT][d]
	constexpr int G = 256 / LANES;
	constexpr int EPG = kRouterTT * kRouterET / G;  // experts per group
	const int t0 = blockIdx.x * kRouterTT;
	const int e0 = blockIdx.y * kRouterET;

	// stage the token tile (rows past T are zero; never written back)
	for (int i = threadIdx.x; i < kRouterTT * d; i += blockDim.x) {
		int tt = i / d, k = i - tt * d;
		xs[i] = (t0 + tt < T) ? x[(int64_t)(t0 + tt) * d + k] : 0.0f;
	}
	__syncthreads();

	const int g = threadIdx.x / LANES;
	const int j = threadIdx.x % LANES;
	const int tt = g % kRouterTT;
	const int eb = (g / kRouterTT) * EPG;
	const float *xr = xs + tt * d;

	const float *wr[EPG];
	float acc[EPG];
#pragma unroll
	for (int q = 0; q < EPG; q++) {
		int e = min(e0 + eb + q, NE - 1);
		wr[q] = w + (int64_t)e * d;
		acc[q] = 0.0f;
	}
	const int nv = d - d % LANES;
	for (int i = j; i < nv; i += LANES) {
		float xv = xr[i];
#pragma unroll
		for (int q = 0; q < EPG; q++)
			acc[q] = __fmaf_rn(xv, __ldg(wr[q] + i), acc[q]);
	}
#pragma unroll
	for (int q = 0; q < EPG; q++) {
		float s = lane_tree_sum<LANES>(acc[q]);
		if (j == 0) {
			// matmul.c:97-104 scalar tail, contracted to FMA by gcc -O3
			for (int i = nv; i < d; i++)
				s = __fmaf_rn(xr[i], wr[q][i], s);
			int e = e0 + eb + q;
			if (t0 + tt < T && e < NE)
				logits[(int64_t)(t0 + tt) * NE + e] = __fadd_rn(0.0f, s);
		}
	}
}

// ---------------------------------------------------------------------
// Tiled router logits (d % 256 == 0, NE % 16 == 0).  Same FMA chains as
// router_logits_kernel, but each thread keeps four consecutive SIMD lanes
// (one lane quad) for a TQ x EQ (token x expert) register tile, so every
// float4 it reads from shared memory feeds 4*EQ (or 4*TQ) FMAs.  The CTA
// tile is TT tokens x 16 experts; d is staged 256 columns at a time.
// The lane tree (upper half onto lower half) becomes a shuffle with the
// thread two (then one) quads away, then two in-register adds.
// CTAs of the first expert tile also write the fp16 hi/lo split of x that
// the expert kernels read (Q4_0: block-permuted, see q4_src).
// ---------------------------------------------------------------------
constexpr int kRChunk = 256;
constexpr int kRET = 16;

__device__ __forceinline__ int q4_src_dev(int k)
{
	const int base = k & ~31, c = (k & 31) >> 3, j = k & 7;
	return base + 4 * c + 16 * ((j >> 1) & 1) + ((j >> 2) & 1) + 2 * (j & 1);
}

template <int LANES, int TQ, int EQ, int TT, int CH>
__global__ void __launch_bounds__(256)
router_tiled_kernel(const float *__restrict__ x, const float *__restrict__ w,
		    float *__restrict__ logits, int T, int d, int NE,
		    __half *__restrict__ x16, int q4)
{
	constexpr int LQ = LANES / 4;                 // lane quads per logit
	constexpr int EG = kRET / EQ;                 // expert groups per CTA
	constexpr int TG = TT / TQ;                   // token groups per CTA
	static_assert(LQ * EG * TG == 256, "one thread per (lane quad, token grp, expert grp)");
	constexpr int XV = TT * CH / 4 / 256;         // float4 per thread to stage x
	constexpr int WV = kRET * CH / 4 / 256;       // float4 per thread to stage w
	static_assert(XV >= 1 && WV >= 1, "tile too small for 256 threads");
	extern __shared__ __align__(16) float rsm[];
	float(*xs)[CH] = reinterpret_cast<float(*)[CH]>(rsm);             // [TT][CH]
	float(*ws)[CH] = reinterpret_cast<float(*)[CH]>(rsm + TT * CH);   // [16][CH]

	const int tid = threadIdx.x;
	const int lq = tid % LQ, combo = tid / LQ;
	const int tg = combo % TG, eg = combo / TG;
	const int t0 = blockIdx.x * TT, e0 = blockIdx.y * kRET;
	const bool write16 = x16 != nullptr && blockIdx.y == 0;

	float acc[TQ][EQ][4];
#pragma unroll
	for (int a = 0; a < TQ; a++)
#pragma unroll
		for (int b = 0; b < EQ; b++)
#pragma unroll
			for (int j = 0; j < 4; j++)
				acc[a][b][j] = 0.0f;

	// register staging of the next chunk (global latency overlaps compute)
	float4 xr[XV], wr[WV];
	auto fetch = [&](int c0) {
#pragma unroll
		for (int v = 0; v < XV; v++) {
			const int i = tid + v * 256, tt = i / (CH / 4), k4 = i % (CH / 4);
			xr[v] = (t0 + tt < T) ? __ldg(reinterpret_cast<const float4 *>(
							    x + (int64_t)(t0 + tt) * d + c0) + k4)
					      : make_float4(0.f, 0.f, 0.f, 0.f);
		}
#pragma unroll
		for (int v = 0; v < WV; v++) {
			const int i = tid + v * 256, ee = i / (CH / 4), k4 = i % (CH / 4);
			wr[v] = __ldg(reinterpret_cast<const float4 *>(w + (int64_t)(e0 + ee) * d + c0) + k4);
		}
	};
	auto store = [&]() {
#pragma unroll
		for (int v = 0; v < XV; v++) {
			const int i = tid + v * 256;
			reinterpret_cast<float4 *>(xs[i / (CH / 4)])[i % (CH / 4)] = xr[v];
		}
#pragma unroll
		for (int v = 0; v < WV; v++) {
			const int i = tid + v * 256;
			reinterpret_cast<float4 *>(ws[i / (CH / 4)])[i % (CH / 4)] = wr[v];
		}
	};

	fetch(0);
	store();
	__syncthreads();
	for (int c0 = 0; c0 < d; c0 += CH) {
		const bool more = c0 + CH < d;
		if (more)
			fetch(c0 + CH);
		if (write16) {
			for (int i = tid; i < TT * CH; i += 256) {
				const int tt = i / CH, k = i % CH;
				if (t0 + tt >= T)
					continue;
				const float v = xs[tt][q4 ? q4_src_dev(k) : k];
				const __half h = __float2half_rn(v);
				__half *o = x16 + (int64_t)(t0 + tt) * 2 * d + c0 + k;
				o[0] = h;
				o[d] = __float2half_rn(__fsub_rn(v, __half2float(h)));
			}
		}
#pragma unroll 4
		for (int s = 0; s < CH / LANES; s++) {
			const int col = s * LANES + lq * 4;
			float4 xv[TQ], wv[EQ];
#pragma unroll
			for (int a = 0; a < TQ; a++)
				xv[a] = *reinterpret_cast<const float4 *>(&xs[tg * TQ + a][col]);
#pragma unroll
			for (int b = 0; b < EQ; b++)
				wv[b] = *reinterpret_cast<const float4 *>(&ws[eg * EQ + b][col]);
#pragma unroll
			for (int a = 0; a < TQ; a++)
#pragma unroll
				for (int b = 0; b < EQ; b++) {
					acc[a][b][0] = __fmaf_rn(xv[a].x, wv[b].x, acc[a][b][0]);
					acc[a][b][1] = __fmaf_rn(xv[a].y, wv[b].y, acc[a][b][1]);
					acc[a][b][2] = __fmaf_rn(xv[a].z, wv[b].z, acc[a][b][2]);
					acc[a][b][3] = __fmaf_rn(xv[a].w, wv[b].w, acc[a][b][3]);
				}
		}
		if (more) {
			__syncthreads();  // everyone is done reading this chunk
			store();
			__syncthreads();
		}
	}
	// lane tree: quads live in consecutive threads (lq = tid % LQ)
#pragma unroll
	for (int a = 0; a < TQ; a++)
#pragma unroll
		for (int b = 0; b < EQ; b++) {
			float *v = acc[a][b];
			if (LQ == 4) {
				// lanes j += j+8  ==  quad lq += quad lq+2
#pragma unroll
				for (int j = 0; j < 4; j++)
					v[j] = __fadd_rn(v[j], __shfl_down_sync(0xffffffffu, v[j], 2, 4));
			}
			// lanes j += j+4  ==  quad lq += quad lq+1
#pragma unroll
			for (int j = 0; j < 4; j++)
				v[j] = __fadd_rn(v[j], __shfl_down_sync(0xffffffffu, v[j], 1, LQ));
			const float s = __fadd_rn(__fadd_rn(v[0], v[2]), __fadd_rn(v[1], v[3]));
			const int t = t0 + tg * TQ + a, e = e0 + eg * EQ + b;
			if (lq == 0 && t < T)
				logits[(int64_t)t * NE + e] = __fadd_rn(0.0f, s);
		}
}

constexpr int kTopkWarps = 4;

template <int LANES>
__global__ void __launch_bounds__(32 * kTopkWarps)
router_topk_kernel(const float *__restrict__ logits, const float *__restrict__ bias,
		   int T, int NE, int K, int mode_exact, int renorm,
		   int32_t *__restrict__ ids, float *__restrict__ wts, float *__restrict__ probs_out)
{
	extern __shared__ float sm[];  // [kTopkWarps][2K] selected weights and ids
	const int warp = threadIdx.x / 32;
	const int t = blockIdx.x * kTopkWarps + warp;
	if (t >= T)
		return;  // whole warp leaves together
	float *sw = sm + warp * 2 * K;
	topk_token<LANES>(logits + (int64_t)t * NE, bias, NE, K, mode_exact, renorm,
			  sw, reinterpret_cast<int32_t *>(sw + K), ids + (int64_t)t * K,
			  wts + (int64_t)t * K, probs_out ? probs_out + (int64_t)t * NE : nullptr,
			  nullptr);
}

constexpr int kDispatchThreads = 1024;

__global__ void __launch_bounds__(kDispatchThreads)
dispatch_kernel(const int32_t *__restrict__ ids, int npairs, int NE, int first, int nlocal,
		int32_t *__restrict__ counts, int32_t *__restrict__ offsets,
		int32_t *__restrict__ perm, int32_t *__restrict__ pos_of,
		int32_t *__restrict__ active, int32_t *__restrict__ n_active,
		int32_t *__restrict__ err, int32_t *__restrict__ work)
{
	extern __shared__ int32_t ds[];
	if (threadIdx.x == 0)
		work[0] = work[1] = 0;
	dispatch_body(ids, npairs, NE, first, nlocal, counts, offsets, perm, pos_of, active,
		      n_active, err, ds);
}

// small batches: softmax/top-k of every token (warp w takes tokens w,
// w+32, ...) and the dispatch in one CTA, ids kept in shared memory.
// smem: sel [32][2K], ids [T*K], dispatch scratch
template <int LANES>
__global__ void __launch_bounds__(kDispatchThreads)
route_small_kernel(const float *__restrict__ logits, const float *__restrict__ bias, int T,
		   int NE, int K, int mode_exact, int renorm, int first, int nlocal,
		   int32_t *__restrict__ ids, float *__restrict__ wts,
		   int32_t *__restrict__ counts, int32_t *__restrict__ offsets,
		   int32_t *__restrict__ perm, int32_t *__restrict__ pos_of,
		   int32_t *__restrict__ active, int32_t *__restrict__ n_active,
		   int32_t *__restrict__ err, int32_t *__restrict__ work)
{
	extern __shared__ float rs[];
	const int warp = threadIdx.x / 32;
	float *sel = rs;                                     // [32][2K]
	int32_t *ids_s = reinterpret_cast<int32_t *>(sel + 64 * K);  // [T*K]
	int32_t *ds = ids_s + T * K;
	if (threadIdx.x == 0)
		work[0] = work[1] = 0;
	for (int t = warp; t < T; t += 32) {
		float *sw = sel + warp * 2 * K;
		topk_token<LANES>(logits + (int64_t)t * NE, bias, NE, K, mode_exact, renorm,
				  sw, reinterpret_cast<int32_t *>(sw + K),
				  ids + (int64_t)t * K, wts + (int64_t)t * K, nullptr, ids_s + t * K);
	}
	__syncthreads();
	dispatch_body(ids_s, T * K, NE, first, nlocal, counts, offsets, perm, pos_of, active,
		      n_active, err, ds);
}

// One token (T = 1): the router logit of expert blockIdx.x by one warp (the
// same LANES-lane chains and halving tree as the kernels above, both rows
// staged in shared memory by the whole CTA first), then the last CTA to
// finish ranks the token's experts (topk_tokens_cta) and dispatches its K
// pairs (dispatch_warp).  cnt: an arrival counter, zero at launch and
// reset by the last CTA.  smem: x [d], the expert's row [d], top-k scratch.
constexpr int kT1Threads = 64;

template <int LANES>
__global__ void __launch_bounds__(kT1Threads)
router_t1_kernel(const float *__restrict__ x, const float *__restrict__ w,
		 const float *__restrict__ bias, int d, int NE, int K, int mode_exact, int renorm,
		 float *__restrict__ logits, int32_t *__restrict__ ids, float *__restrict__ wts,
		 int32_t *__restrict__ counts, int32_t *__restrict__ offsets,
		 int32_t *__restrict__ perm, int32_t *__restrict__ pos_of,
		 int32_t *__restrict__ active, int32_t *__restrict__ n_active,
		 int32_t *__restrict__ err, int32_t *__restrict__ work, unsigned *cnt)
{
	extern __shared__ __align__(16) float rs[];
	__shared__ int last;
	// the expert GEMVs after it may start their set-up (they wait for the
	// routing before reading it)
	griddep_launch_dependents();
	const int tid = threadIdx.x, e = blockIdx.x;
	const float4 *x4 = reinterpret_cast<const float4 *>(x);
	const float4 *w4 = reinterpret_cast<const float4 *>(w + (int64_t)e * d);
	float4 *sx = reinterpret_cast<float4 *>(rs), *sw = reinterpret_cast<float4 *>(rs + d);
	for (int i = tid; i < d / 4; i += blockDim.x) {
		sx[i] = __ldg(x4 + i);
		sw[i] = __ldg(w4 + i);
	}
	__syncthreads();
	if (tid < 32) {
		// lane q < LANES / 4 carries SIMD lanes 4q..4q+3: element
		// st * LANES + 4q + c goes to chain 4q + c, in order of st
		constexpr int Q = LANES / 4;
		float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
		if (tid < Q) {
#pragma unroll 8
			for (int st = 0; st < d / LANES; st++) {
				const float4 xv = sx[st * Q + tid], wv = sw[st * Q + tid];
				a0 = __fmaf_rn(xv.x, wv.x, a0);
				a1 = __fmaf_rn(xv.y, wv.y, a1);
				a2 = __fmaf_rn(xv.z, wv.z, a2);
				a3 = __fmaf_rn(xv.w, wv.w, a3);
			}
		}
		float l[LANES];
#pragma unroll
		for (int q = 0; q < Q; q++) {
			l[4 * q] = __shfl_sync(0xffffffffu, a0, q);
			l[4 * q + 1] = __shfl_sync(0xffffffffu, a1, q);
			l[4 * q + 2] = __shfl_sync(0xffffffffu, a2, q);
			l[4 * q + 3] = __shfl_sync(0xffffffffu, a3, q);
		}
#pragma unroll
		for (int h = LANES / 2; h >= 1; h /= 2)
#pragma unroll
			for (int j = 0; j < h; j++)
				l[j] = __fadd_rn(l[j], l[j + h]);
		if (tid == 0)
			logits[e] = __fadd_rn(0.0f, l[0]);
	}
	if (tid == 0) {
		__threadfence();
		last = atomicAdd(cnt, 1u) == (unsigned)NE - 1;
	}
	__syncthreads();
	if (!last)
		return;
	__threadfence();
	float *scr = rs + 2 * d;                                      // 64 + LANES + 1 + 2K
	int32_t *ids_s = reinterpret_cast<int32_t *>(scr + 64 + LANES + 1 + 2 * K);  // [K]
	float *w_s = reinterpret_cast<float *>(ids_s + K);            // [K]
	topk_tokens_cta<LANES>(logits, bias, 1, NE, K, mode_exact, renorm, scr, ids_s, w_s, ids, wts);
	__syncthreads();
	if (tid < 32) {
		dispatch_warp(ids_s, K, NE, 0, NE, counts, offsets, perm, active, n_active, err);
		if (tid < K) {
			const int p = perm[tid];
			if (p >= 0 && p < K)
				pos_of[p] = tid;
		}
	}
	if (tid == 0) {
		work[0] = work[1] = 0;
		*cnt = 0u;
	}
}

// ---------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------
bool router_t1_ok(int d, int NE, int K)
{
	return d % 64 == 0 && d <= 16384 && NE >= 1 && NE <= 64 && K >= 1 && K <= NE && K <= 32;
}

cudaError_t launch_router_t1(const float *x, const float *w, const float *bias, int d, int NE,
			     int K, int lanes, int mode_exact, int renorm, float *logits,
			     int32_t *ids, float *wts, int32_t *counts, int32_t *offsets,
			     int32_t *perm, int32_t *pos_of, int32_t *active, int32_t *n_active,
			     int32_t *err, int32_t *work, unsigned *cnt, cudaStream_t st)
{
	if (!router_t1_ok(d, NE, K))
		return cudaErrorNotSupported;
	const size_t smem = ((size_t)2 * d + 64 + 16 + 1 + 4 * K) * sizeof(float);
	auto fn = lanes == 8 ? router_t1_kernel<8> : router_t1_kernel<16>;
	cudaError_t e = ensure_smem(fn, smem);
	if (e != cudaSuccess)
		return e;
	fn<<<NE, kT1Threads, smem, st>>>(x, w, bias, d, NE, K, mode_exact, renorm, logits, ids, wts,
					 counts, offsets, perm, pos_of, active, n_active, err, work,
					 cnt);
	return cudaGetLastError();
}
template <int LANES, int TQ, int EQ, int TT, int CH>
static cudaError_t run_tiled(const float *x, const float *w, float *logits, int T, int d, int NE,
			     __half *x16, int q4, cudaStream_t st)
{
	const size_t smem = (size_t)(TT + kRET) * CH * sizeof(float);
	auto fn = router_tiled_kernel<LANES, TQ, EQ, TT, CH>;
	cudaError_t e = ensure_smem(fn, smem);
	if (e != cudaSuccess)
		return e;
	fn<<<dim3((T + TT - 1) / TT, NE / kRET), 256, smem, st>>>(x, w, logits, T, d, NE, x16, q4);
	return cudaGetLastError();
}

cudaError_t launch_router_tiled(const float *x, const float *w, int T, int d, int NE, int lanes,
				float *logits, __half *x16, int q4, cudaStream_t st)
{
	if (T == 0 || NE == 0)
		return cudaSuccess;
	// decode-sized batches: one logit (lane quad) per thread, 4-8 tokens per
	// CTA so that many CTAs share the work; prefill: 4x4 register tiles
	const bool big = T > 128;
	if (lanes == 8) {
		if (big)
			return run_tiled<8, 2, 4, 64, 256>(x, w, logits, T, d, NE, x16, q4, st);
		return run_tiled<8, 1, 1, 8, 256>(x, w, logits, T, d, NE, x16, q4, st);
	}
	if (big)
		return run_tiled<16, 4, 4, 64, 256>(x, w, logits, T, d, NE, x16, q4, st);
	return run_tiled<16, 1, 1, 4, 256>(x, w, logits, T, d, NE, x16, q4, st);
}

bool router_tiled_ok(int d, int NE)
{
	return d % kRChunk == 0 && NE % kRET == 0;
}

cudaError_t launch_router_logits(const float *x, const float *w, int T, int d, int NE, int lanes,
				 float *logits, cudaStream_t st)
{
	if (T == 0 || NE == 0)
		return cudaSuccess;
	dim3 grid((T + kRouterTT - 1) / kRouterTT, (NE + kRouterET - 1) / kRouterET);
	size_t smem = (size_t)kRouterTT * d * sizeof(float);
	cudaError_t e;
	if (lanes == 8) {
		e = ensure_smem(router_logits_kernel<8>, smem);
		if (e != cudaSuccess)
			return e;
		router_logits_kernel<8><<<grid, 256, smem, st>>>(x, w, logits, T, d, NE);
	} else {
		e = ensure_smem(router_logits_kernel<16>, smem);
		if (e != cudaSuccess)
			return e;
		router_logits_kernel<16><<<grid, 256, smem, st>>>(x, w, logits, T, d, NE);
	}
	return cudaGetLastError();
}

cudaError_t launch_router_topk(const float *logits, const float *bias, int T, int NE, int K,
			       int lanes, int mode_exact, int renorm, int32_t *ids, float *wts,
			       float *probs, cudaStream_t st)
{
	if (T == 0)
		return cudaSuccess;
	const int blocks = (T + kTopkWarps - 1) / kTopkWarps;
	const size_t tsm = (size_t)kTopkWarps * 2 * K * sizeof(float);
	if (lanes == 8)
		router_topk_kernel<8><<<blocks, 32 * kTopkWarps, tsm, st>>>(
			logits, bias, T, NE, K, mode_exact, renorm, ids, wts, probs);
	else
		router_topk_kernel<16><<<blocks, 32 * kTopkWarps, tsm, st>>>(
			logits, bias, T, NE, K, mode_exact, renorm, ids, wts, probs);
	return cudaGetLastError();
}

cudaError_t launch_router(const float *x, const float *w, const float *bias, int T, int d,
			  int NE, int K, int lanes, int mode_exact, int renorm, float *logits,
			  int32_t *ids, float *wts, float *probs, cudaStream_t st)
{
	cudaError_t e = launch_router_logits(x, w, T, d, NE, lanes, logits, st);
	if (e != cudaSuccess)
		return e;
	return launch_router_topk(logits, bias, T, NE, K, lanes, mode_exact, renorm, ids, wts,
				  probs, st);
}

static size_t dispatch_smem(int NE) { return (size_t)(2 * NE + 32 * NE) * sizeof(int32_t); }

cudaError_t launch_dispatch(const int32_t *ids, int npairs, int NE, int first, int nlocal,
			    int32_t *counts, int32_t *offsets, int32_t *perm, int32_t *pos_of,
			    int32_t *active, int32_t *n_active, int32_t *err, int32_t *work,
			    cudaStream_t st)
{
	const size_t smem = dispatch_smem(NE);
	cudaError_t e = ensure_smem(dispatch_kernel, smem);
	if (e != cudaSuccess)
		return e;
	dispatch_kernel<<<1, kDispatchThreads, smem, st>>>(ids, npairs, NE, first, nlocal, counts,
							    offsets, perm, pos_of, active, n_active,
							    err, work);
	return cudaGetLastError();
}

size_t route_small_smem(int T, int NE, int K)
{
	return (size_t)(64 * K) * sizeof(float) + (size_t)T * K * sizeof(int32_t) +
	       dispatch_smem(NE);
}

cudaError_t launch_route_small(const float *logits, const float *bias, int T, int NE, int K,
			       int lanes, int mode_exact, int renorm, int first, int nlocal,
			       int32_t *ids, float *wts, int32_t *counts, int32_t *offsets,
			       int32_t *perm, int32_t *pos_of, int32_t *active, int32_t *n_active,
			       int32_t *err, int32_t *work, cudaStream_t st)
{
	const size_t smem = route_small_smem(T, NE, K);
	auto fn = lanes == 8 ? route_small_kernel<8> : route_small_kernel<16>;
	cudaError_t e = ensure_smem(fn, smem);
	if (e != cudaSuccess)
		return e;
	fn<<<1, kDispatchThreads, smem, st>>>(logits, bias, T, NE, K, mode_exact, renorm, first,
					       nlocal, ids, wts, counts, offsets, perm, pos_of,
					       active, n_active, err, work);
	return cudaGetLastError();
}

}  // namespace moe
