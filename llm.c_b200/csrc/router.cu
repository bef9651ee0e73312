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
// softmax + top-k (+ optional renorm), one warp per token.
// ---------------------------------------------------------------------
constexpr int kTopkWarps = 4;

template <int LANES>
__global__ void __launch_bounds__(32 * kTopkWarps)
router_topk_kernel(const float *__restrict__ logits, const float *__restrict__ bias,
		   int T, int NE, int K, int mode_exact, int renorm,
		   int32_t *__restrict__ ids, float *__restrict__ wts, float *__restrict__ probs_out)
{
	extern __shared__ float sm[];  // [kTopkWarps][NE] probs, then [kTopkWarps][2K]
	const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
	const int t = blockIdx.x * kTopkWarps + warp;
	if (t >= T)
		return;  // whole warp leaves together
	float *p = sm + warp * NE;
	const float *lr = logits + (int64_t)t * NE;

	float mx = -INFINITY;
	for (int e = lane; e < NE; e += 32) {
		float v = lr[e];
		if (bias)
			v = __fadd_rn(v, bias[e]);
		p[e] = v;
		mx = fmaxf(mx, v);
	}
	mx = warp_max(mx);
	__syncwarp();
	for (int e = lane; e < NE; e += 32)
		p[e] = exp_rn(__fsub_rn(p[e], mx));
	__syncwarp();

	// lane-wise sums over the vector part (nn.c:236-246), then the tree,
	// then the scalar tail (nn.c:247-250)
	const int nv = NE - NE % LANES;
	float s = 0.0f;
	if (lane < LANES)
		for (int e = lane; e < nv; e += LANES)
			s = __fadd_rn(s, p[e]);
	s = lane_tree_sum<LANES>(s);
	if (lane == 0)
		for (int e = nv; e < NE; e++)
			s = __fadd_rn(s, p[e]);
	s = __shfl_sync(0xffffffffu, s, 0);
	for (int e = lane; e < NE; e += 32)
		p[e] = __fdiv_rn(p[e], s);
	__syncwarp();

	if (probs_out)
		for (int e = lane; e < NE; e += 32)
			probs_out[(int64_t)t * NE + e] = p[e];

	// selections land in shared memory first so lane 0 can renormalise
	float *sw = sm + kTopkWarps * NE + warp * 2 * K;
	int32_t *sid = reinterpret_cast<int32_t *>(sw + K);
	const float p0 = p[0];
	for (int i = lane; i < NE; i += 32) {
		const float v = p[i];
		int rank = 0;
		if (mode_exact) {
			for (int j = 0; j < NE; j++) {
				float o = p[j];
				rank += (o > v) || (o == v && j < i);
			}
			if (rank < K) {
				sid[K - 1 - rank] = i;
				sw[K - 1 - rank] = v;
			}
		} else if (i == 0) {
			// the k seeded copies of element 0
			int r0 = 0;
			for (int j = 1; j < NE; j++)
				r0 += (p[j] > p0);
			for (int c = 0; r0 + c < K; c++) {
				sid[K - 1 - (r0 + c)] = 0;
				sw[K - 1 - (r0 + c)] = p0;
			}
		} else {
			rank = (p0 >= v) ? K : 0;
			for (int j = 1; j < NE && rank < K; j++) {
				float o = p[j];
				rank += (o > v) || (o == v && j < i);
			}
			if (rank < K) {
				sid[K - 1 - rank] = i;
				sw[K - 1 - rank] = v;
			}
		}
	}
	__syncwarp();
	if (renorm && lane == 0) {
		// llama.c:422-427: sequential sum in slot order, then divide
		float sum = 0.0f;
		for (int q = 0; q < K; q++)
			sum = __fadd_rn(sum, sw[q]);
		for (int q = 0; q < K; q++)
			sw[q] = __fdiv_rn(sw[q], sum);
	}
	__syncwarp();
	for (int q = lane; q < K; q += 32) {
		ids[(int64_t)t * K + q] = sid[q];
		wts[(int64_t)t * K + q] = sw[q];
	}
}

// ---------------------------------------------------------------------
// dispatch: counts[NE], offsets[NE+1], perm[T*K] (pairs p = t*K + slot
// stably sorted by expert), pos_of[p] = position of pair p in perm.
// One CTA of 1024 threads walks the pairs in chunks of 1024; within a
// chunk a pair's rank among same-expert pairs comes from warp match masks
// plus per-warp counts, so the order is stable and deterministic.
// ---------------------------------------------------------------------
constexpr int kDispatchThreads = 1024;

__global__ void __launch_bounds__(kDispatchThreads)
dispatch_kernel(const int32_t *__restrict__ ids, int npairs, int NE,
		int32_t *__restrict__ counts, int32_t *__restrict__ offsets,
		int32_t *__restrict__ perm, int32_t *__restrict__ pos_of,
		int32_t *__restrict__ err)
{
	extern __shared__ int32_t ds[];
	int32_t *cnt = ds;                // [NE]
	int32_t *run = cnt + NE;          // [NE] running fill position
	int32_t *wcnt = run + NE;         // [32 warps][NE]
	const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;

	for (int e = tid; e < NE; e += blockDim.x)
		cnt[e] = 0;
	__syncthreads();
	for (int p = tid; p < npairs; p += blockDim.x) {
		int e = ids[p];
		if (e < 0 || e >= NE) {
			atomicExch(err, 1);
			continue;
		}
		atomicAdd(&cnt[e], 1);
	}
	__syncthreads();
	if (tid == 0) {
		int acc = 0;
		for (int e = 0; e < NE; e++) {
			offsets[e] = acc;
			run[e] = acc;
			counts[e] = cnt[e];
			acc += cnt[e];
		}
		offsets[NE] = acc;
	}
	__syncthreads();

	for (int base = 0; base < npairs; base += blockDim.x) {
		for (int i = tid; i < 32 * NE; i += blockDim.x)
			wcnt[i] = 0;
		__syncthreads();
		const int p = base + tid;
		int e = (p < npairs) ? ids[p] : -1;
		if (e >= NE)
			e = -1;
		const unsigned same = __match_any_sync(0xffffffffu, e);
		const int rank_w = __popc(same & ((1u << lane) - 1u));
		if (e >= 0 && rank_w == 0)
			wcnt[warp * NE + e] = __popc(same);
		__syncthreads();
		if (e >= 0) {
			int before = 0;
			for (int w = 0; w < warp; w++)
				before += wcnt[w * NE + e];
			int pos = run[e] + before + rank_w;
			perm[pos] = p;
			if (pos_of)
				pos_of[p] = pos;
		}
		__syncthreads();
		for (int e2 = tid; e2 < NE; e2 += blockDim.x) {
			int add = 0;
			for (int w = 0; w < 32; w++)
				add += wcnt[w * NE + e2];
			run[e2] += add;
		}
		__syncthreads();
	}
}

// ---------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------
cudaError_t launch_router_logits(const float *x, const float *w, int T, int d, int NE, int lanes,
				 float *logits, cudaStream_t st)
{
	if (T == 0 || NE == 0)
		return cudaSuccess;
	dim3 grid((T + kRouterTT - 1) / kRouterTT, (NE + kRouterET - 1) / kRouterET);
	size_t smem = (size_t)kRouterTT * d * sizeof(float);
	cudaError_t e;
	if (lanes == 8) {
		e = cudaFuncSetAttribute(router_logits_kernel<8>,
					 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
		if (e != cudaSuccess)
			return e;
		router_logits_kernel<8><<<grid, 256, smem, st>>>(x, w, logits, T, d, NE);
	} else {
		e = cudaFuncSetAttribute(router_logits_kernel<16>,
					 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
		if (e != cudaSuccess)
			return e;
		router_logits_kernel<16><<<grid, 256, smem, st>>>(x, w, logits, T, d, NE);
	}
	return cudaGetLastError();
}

cudaError_t launch_router(const float *x, const float *w, const float *bias, int T, int d,
			  int NE, int K, int lanes, int mode_exact, int renorm, float *logits,
			  int32_t *ids, float *wts, float *probs, cudaStream_t st)
{
	cudaError_t e = launch_router_logits(x, w, T, d, NE, lanes, logits, st);
	if (e != cudaSuccess || T == 0)
		return e;
	int blocks = (T + kTopkWarps - 1) / kTopkWarps;
	size_t tsm = (size_t)kTopkWarps * (NE + 2 * K) * sizeof(float);
	if (lanes == 8)
		router_topk_kernel<8><<<blocks, 32 * kTopkWarps, tsm, st>>>(
			logits, bias, T, NE, K, mode_exact, renorm, ids, wts, probs);
	else
		router_topk_kernel<16><<<blocks, 32 * kTopkWarps, tsm, st>>>(
			logits, bias, T, NE, K, mode_exact, renorm, ids, wts, probs);
	return cudaGetLastError();
}

cudaError_t launch_dispatch(const int32_t *ids, int npairs, int NE, int32_t *counts,
			    int32_t *offsets, int32_t *perm, int32_t *pos_of, int32_t *err,
			    cudaStream_t st)
{
	size_t smem = (size_t)(2 * NE + 32 * NE) * sizeof(int32_t);
	cudaFuncSetAttribute(dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
			     (int)smem);
	dispatch_kernel<<<1, kDispatchThreads, smem, st>>>(ids, npairs, NE, counts, offsets,
							    perm, pos_of, err);
	return cudaGetLastError();
}

}  // namespace moe
