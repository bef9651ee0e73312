// route_core.cuh — per-token softmax + top-k and the stable expert dispatch,
// shared by the routing kernels (router.cu) and the fused decode-layer
// kernel (decode.cu).
#pragma once

#include "common.cuh"

namespace moe {

constexpr int kMaxTopkExperts = 256;  // experts per router (NE)

// ---------------------------------------------------------------------
// softmax + top-k (+ optional renorm) of one token by one warp, with the
// token's NE probabilities held in registers (element lane + 32 j in v[j]).
// sw/sid: K floats / ints of shared scratch (the selected slots).
// ---------------------------------------------------------------------
template <int LANES, int MAXJ>
static __device__ __noinline__ void topk_token_j(const float *__restrict__ lr, const float *__restrict__ bias,
				    int NE, int K, int mode_exact, int renorm, float *sw, int32_t *sid,
				    int32_t *__restrict__ ids_out, float *__restrict__ w_out,
				    float *__restrict__ probs_out, int32_t *ids_smem)
{
	static_assert(MAXJ * 32 <= kMaxTopkExperts, "register slots per lane");
	constexpr unsigned FULL = 0xffffffffu;
	const int lane = threadIdx.x % 32;
	const int nj = (NE + 31) / 32;
	float v[MAXJ];
	float mx = -INFINITY;
#pragma unroll
	for (int j = 0; j < MAXJ; j++) {
		const int e = lane + 32 * j;
		v[j] = 0.0f;
		if (j < nj && e < NE) {
			float l = lr[e];
			if (bias)
				l = __fadd_rn(l, bias[e]);
			v[j] = l;
			mx = fmaxf(mx, l);
		}
	}
	mx = warp_max(mx);
#pragma unroll
	for (int j = 0; j < MAXJ; j++)
		if (j < nj && lane + 32 * j < NE)
			v[j] = exp_rn(__fsub_rn(v[j], mx));

	// nn.c:236-250: SIMD lane l (< LANES) sums elements l, l+LANES, l+2 LANES,
	// ... of the vector part in order; the lanes meet in the halving tree;
	// the scalar tail is added after it, in order
	const int nv = NE - NE % LANES;
	float s = 0.0f;
#pragma unroll
	for (int m = 0; m < MAXJ * 32 / LANES; m++) {
		// element lane + LANES*m lives in lane lane + (LANES*m % 32), slot LANES*m / 32
		const float o = __shfl_sync(FULL, v[(LANES * m) / 32], lane + (LANES * m) % 32);
		if (m < nv / LANES)
			s = __fadd_rn(s, o);
	}
	s = lane_tree_sum<LANES>(s);
	for (int e = nv; e < NE; e++) {
		float o = 0.0f;
#pragma unroll
		for (int j = 0; j < MAXJ; j++)
			if (e / 32 == j)
				o = __shfl_sync(FULL, v[j], e & 31);
		s = __fadd_rn(s, o);  // lane 0's value is the reference's
	}
	s = __shfl_sync(FULL, s, 0);
#pragma unroll
	for (int j = 0; j < MAXJ; j++)
		if (j < nj && lane + 32 * j < NE) {
			v[j] = __fdiv_rn(v[j], s);
			if (probs_out)
				probs_out[lane + 32 * j] = v[j];
		}

	// Reference mode: nn.c:276-308 seeds all k slots with element 0, which
	// equals ranking [p0 (k copies), p1, p2, ...] by (value desc, position
	// asc): the result is, in rank order, the elements ahead of element 0 in
	// the (value desc, index asc) order (at most k of them), then copies of
	// element 0 (weight p0).  Exact mode: the first k of that order.
	// Slot of rank r = K-1-r.
	const float p0 = __shfl_sync(FULL, v[0], 0);
	if constexpr (MAXJ == 2) {
		// NE <= 64: bitonic sort of the 64 (value, index) keys, descending,
		// positions lane and lane + 32 (padding sorts last)
		float kv[2];
		int ki[2];
#pragma unroll
		for (int s = 0; s < 2; s++) {
			ki[s] = lane + 32 * s;
			kv[s] = ki[s] < NE ? v[s] : -1.0f;
		}
		auto first = [](float va, int ia, float vb, int ib) {  // a ahead of b
			return va > vb || (va == vb && ia < ib);
		};
		// rolled loops: this code runs once per token and mostly with a cold
		// instruction cache, so it is kept short
#pragma unroll 1
		for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll 1
			for (int j = k >> 1; j > 0; j >>= 1) {
				if (j == 32) {
					// both positions of the pair live in this lane; the block
					// (k = 64) is descending
					if (!first(kv[0], ki[0], kv[1], ki[1])) {
						const float tv = kv[0];
						const int ti = ki[0];
						kv[0] = kv[1];
						ki[0] = ki[1];
						kv[1] = tv;
						ki[1] = ti;
					}
				} else {
#pragma unroll
					for (int s = 0; s < 2; s++) {
						const int pos = lane + 32 * s;
						const float ov = __shfl_xor_sync(FULL, kv[s], j);
						const int oi = __shfl_xor_sync(FULL, ki[s], j);
						const bool desc = (pos & k) == 0;     // block direction
						const bool lower = (pos & j) == 0;    // lower position of the pair
						const bool mine_first = first(kv[s], ki[s], ov, oi);
						if (mine_first != (lower == desc)) {
							kv[s] = ov;
							ki[s] = oi;
						}
					}
				}
			}
		}
		// rank r sits in lane r (s = 0) for r < 32; element 0's rank q
		const unsigned at0 = __ballot_sync(FULL, ki[0] == 0), at1 = __ballot_sync(FULL, ki[1] == 0);
		const int q = at0 ? __ffs(at0) - 1 : 32 + __ffs(at1) - 1;
#pragma unroll
		for (int s = 0; s < 2; s++) {
			const int rk = lane + 32 * s;  // rank held here
			if (rk < K) {
				const bool copy0 = !mode_exact && rk >= q;
				sid[K - 1 - rk] = copy0 ? 0 : ki[s];
				sw[K - 1 - rk] = copy0 ? p0 : kv[s];
			}
		}
	} else {
		// rank of every element, all at once: element i's rank counts the
		// elements ahead of it by (value desc, index asc); in reference mode
		// element i >= 1 starts behind the k copies when p0 >= p_i, and
		// element 0 fills slots r0 .. k-1 where r0 = #{j >= 1 : p_j > p0}.
		int rank[MAXJ];
#pragma unroll
		for (int j = 0; j < MAXJ; j++)
			rank[j] = (!mode_exact && p0 >= v[j]) ? K : 0;
		int r0 = 0;  // reference mode, element 0 (lane 0)
		// Every shuffle is unconditional (a shuffle under a branch costs a
		// reconvergence barrier); validity enters as predicates.
#pragma unroll 8
		for (int l = 0; l < 32; l++) {
#pragma unroll
			for (int jj = 0; jj < MAXJ; jj++) {
				const float o = __shfl_sync(FULL, v[jj], l);
				const int eo = l + 32 * jj;
				const bool cand = eo < NE && (mode_exact || eo != 0);
#pragma unroll
				for (int j = 0; j < MAXJ; j++) {
					const int e = lane + 32 * j;
					rank[j] += cand && (o > v[j] || (o == v[j] && eo < e));
				}
				r0 += eo < NE && eo != 0 && o > p0;
			}
		}
#pragma unroll
		for (int j = 0; j < MAXJ; j++) {
			const int e = lane + 32 * j;
			if (j >= nj || e >= NE) {
			} else if (!mode_exact && e == 0) {
				for (int c = r0; c < K; c++) {
					sid[K - 1 - c] = 0;
					sw[K - 1 - c] = p0;
				}
			} else if (rank[j] < K) {
				sid[K - 1 - rank[j]] = e;
				sw[K - 1 - rank[j]] = v[j];
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
		ids_out[q] = sid[q];
		w_out[q] = sw[q];
		if (ids_smem)
			ids_smem[q] = sid[q];
	}
	__syncwarp();
}

// The same softmax + top-k for T <= blockDim.x / 64 tokens at once, one
// thread per (token, expert) (NE <= 64), for the few-token decode batches
// where a single warp's serial shuffle chain would be the latency: the max,
// the exponentials, the LANES-chain sum with its halving tree and the tail,
// the divisions and the ranks (reference mode or exact) are the same
// operations in the same order as topk_token_j, spread over the CTA.  Every
// thread of the CTA calls it (it synchronises the CTA).  lg: [T][NE]
// logits (global); scr: shared scratch of T * (64 + LANES + 1 + 2 * K)
// words; ids_s/w_s: [T][K] outputs in slot order (shared); ids_g/w_g: the
// same to global memory (or NULL).
template <int LANES>
static __device__ void topk_tokens_cta(const float *__restrict__ lg, const float *__restrict__ bias,
				       int T, int NE, int K, int mode_exact, int renorm, float *scr,
				       int32_t *ids_s, float *w_s, int32_t *ids_g, float *w_g)
{
	float *P = scr;                          // [T][64]
	float *CS = P + T * 64;                  // [T][LANES]
	float *SUM = CS + T * LANES;             // [T]
	int32_t *SID = reinterpret_cast<int32_t *>(SUM + T);  // [T][K]
	float *SW = reinterpret_cast<float *>(SID + T * K);   // [T][K]
	const int tid = threadIdx.x, t = tid / 64, e = tid % 64;
	const bool act = t < T && e < NE;
	float l = 0.0f;
	if (act) {
		l = __ldcg(lg + (int64_t)t * NE + e);
		if (bias)
			l = __fadd_rn(l, bias[e]);
		P[t * 64 + e] = l;
	}
	__syncthreads();
	float v = 0.0f;
	if (act) {
		float mx = -INFINITY;
		for (int i = 0; i < NE; i++)
			mx = fmaxf(mx, P[t * 64 + i]);
		v = exp_rn(__fsub_rn(l, mx));
	}
	__syncthreads();
	if (act)
		P[t * 64 + e] = v;
	__syncthreads();
	// nn.c:236-250: lane c sums elements c, c + LANES, ... of the vector part
	// in order; the halving tree over the lanes; the scalar tail in order
	const int nv = NE - NE % LANES;
	if (t < T && e < LANES) {
		float s = 0.0f;
		for (int m = 0; m < nv / LANES; m++)
			s = __fadd_rn(s, P[t * 64 + e + LANES * m]);
		CS[t * LANES + e] = s;
	}
	__syncthreads();
	if (t < T && e == 0) {
		float c[LANES];
#pragma unroll
		for (int j = 0; j < LANES; j++)
			c[j] = CS[t * LANES + j];
#pragma unroll
		for (int h = LANES / 2; h >= 1; h /= 2)
#pragma unroll
			for (int j = 0; j < h; j++)
				c[j] = __fadd_rn(c[j], c[j + h]);
		float s = c[0];
		for (int i = nv; i < NE; i++)
			s = __fadd_rn(s, P[t * 64 + i]);
		SUM[t] = s;
	}
	__syncthreads();
	const float p = act ? __fdiv_rn(v, SUM[t]) : 0.0f;
	__syncthreads();
	if (act)
		P[t * 64 + e] = p;
	__syncthreads();
	// ranks by (value desc, index asc); reference mode (nn.c:276-308 seeds
	// every slot with element 0): elements not above p0 fall behind its k
	// copies, which fill the slots from r0 = #{i >= 1 : p_i > p0} on
	if (act) {
		const float p0 = P[t * 64];
		if (mode_exact || e != 0) {
			int rank = (!mode_exact && p0 >= p) ? K : 0;
			for (int i = 0; i < NE; i++) {
				const float o = P[t * 64 + i];
				rank += (mode_exact || i != 0) && (o > p || (o == p && i < e));
			}
			if (rank < K) {
				SID[t * K + K - 1 - rank] = e;
				SW[t * K + K - 1 - rank] = p;
			}
		} else {
			int r0 = 0;
			for (int i = 1; i < NE; i++)
				r0 += P[t * 64 + i] > p0;
			for (int c = r0; c < K; c++) {
				SID[t * K + K - 1 - c] = 0;
				SW[t * K + K - 1 - c] = p0;
			}
		}
	}
	__syncthreads();
	if (renorm && t < T && e == 0) {
		// llama.c:422-427: sequential sum in slot order, then divide
		float sum = 0.0f;
		for (int q = 0; q < K; q++)
			sum = __fadd_rn(sum, SW[t * K + q]);
		for (int q = 0; q < K; q++)
			SW[t * K + q] = __fdiv_rn(SW[t * K + q], sum);
	}
	__syncthreads();
	if (t < T && e < K) {
		ids_s[t * K + e] = SID[t * K + e];
		w_s[t * K + e] = SW[t * K + e];
		if (ids_g) {
			ids_g[(int64_t)t * K + e] = SID[t * K + e];
			w_g[(int64_t)t * K + e] = SW[t * K + e];
		}
	}
	__syncthreads();
}

// NE <= 32 * MAXJ elements per token: the smallest register file that fits.
// topk_token_j is kept out of line so that its register arrays stay in
// registers inside large kernels as well.
template <int LANES>
static __device__ void topk_token(const float *__restrict__ lr, const float *__restrict__ bias,
				  int NE, int K, int mode_exact, int renorm, float *sw, int32_t *sid,
				  int32_t *__restrict__ ids_out, float *__restrict__ w_out,
				  float *__restrict__ probs_out, int32_t *ids_smem)
{
	if (NE <= 64)
		topk_token_j<LANES, 2>(lr, bias, NE, K, mode_exact, renorm, sw, sid, ids_out, w_out,
				       probs_out, ids_smem);
	else if (NE <= 128)
		topk_token_j<LANES, 4>(lr, bias, NE, K, mode_exact, renorm, sw, sid, ids_out, w_out,
				       probs_out, ids_smem);
	else
		topk_token_j<LANES, 8>(lr, bias, NE, K, mode_exact, renorm, sw, sid, ids_out, w_out,
				       probs_out, ids_smem);
}

// ---------------------------------------------------------------------
// dispatch: counts[NE], offsets[NE+1], perm[T*K] (pairs p = t*K + slot
// stably sorted by expert), pos_of[p] = position of pair p in perm, and the
// ascending list of experts in [first, first+nlocal) that received pairs.
// One CTA walks the pairs in chunks of blockDim.x; within a chunk a
// pair's rank among same-expert pairs comes from warp match masks plus
// per-warp counts, so the order is stable and deterministic.  Every thread
// of the CTA must call it (it synchronises the CTA).
// smem: cnt[NE], run[NE], wcnt[warps][NE]; blockDim.x a multiple of 32
// ---------------------------------------------------------------------
// The same dispatch for at most 32 pairs, by one warp (lane p holds pair p):
// a pair's position is the number of pairs with a smaller expert id plus
// the earlier pairs with its own, which is dispatch_body's stable order.
// Called by one warp; the caller synchronises the CTA after it.
static __device__ void dispatch_warp(const int32_t *ids, int npairs, int NE, int first, int nlocal,
				     int32_t *__restrict__ counts, int32_t *__restrict__ offsets,
				     int32_t *__restrict__ perm, int32_t *__restrict__ active,
				     int32_t *__restrict__ n_active, int32_t *__restrict__ err)
{
	constexpr unsigned FULL = 0xffffffffu;
	const int lane = threadIdx.x % 32;
	int e = lane < npairs ? ids[lane] : -1;
	if (lane < npairs && (e < 0 || e >= NE)) {
		atomicExch(err, 1);
		e = -1;
	}
	int below = 0, same_before = 0;
	for (int q = 0; q < 32; q++) {
		const int eq = __shfl_sync(FULL, e, q);
		below += eq >= 0 && eq < e;
		same_before += eq == e && q < lane;
	}
	if (e >= 0)
		perm[below + same_before] = lane;
	int na = 0;
	for (int base = 0; base < NE; base += 32) {
		const int x = base + lane;
		int c = 0, o = 0;
		for (int q = 0; q < 32; q++) {
			const int eq = __shfl_sync(FULL, e, q);
			c += eq == x;
			o += eq >= 0 && eq < x;
		}
		if (x < NE) {
			counts[x] = c;
			offsets[x] = o;
		}
		const bool act = x < NE && c > 0 && x >= first && x < first + nlocal;
		const unsigned m = __ballot_sync(FULL, act);
		if (act)
			active[na + __popc(m & ((1u << lane) - 1u))] = x;
		na += __popc(m);
	}
	const unsigned valid = __ballot_sync(FULL, e >= 0);
	if (lane == 0) {
		offsets[NE] = __popc(valid);
		*n_active = na;
	}
	__syncwarp();
}

static __device__ void dispatch_body(const int32_t *ids, int npairs, int NE, int first, int nlocal,
			      int32_t *__restrict__ counts, int32_t *__restrict__ offsets,
			      int32_t *__restrict__ perm, int32_t *__restrict__ pos_of,
			      int32_t *__restrict__ active, int32_t *__restrict__ n_active,
			      int32_t *__restrict__ err, int32_t *ds)
{
	int32_t *cnt = ds;                // [NE]
	int32_t *run = cnt + NE;          // [NE] running fill position
	int32_t *wcnt = run + NE;         // [warps][NE]
	const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
	const int nw = (int)blockDim.x / 32;  // warps of the CTA (at most 32)

	for (int e = tid; e < NE; e += blockDim.x)
		cnt[e] = 0;
	__syncthreads();
	for (int p = tid; p < npairs; p += blockDim.x) {
		const int e = ids[p];
		if (e < 0 || e >= NE) {
			atomicExch(err, 1);
			continue;
		}
		atomicAdd(&cnt[e], 1);
	}
	__syncthreads();
	if (warp == 0) {
		// exclusive scan of the counts and the list of active local experts,
		// 32 experts at a time (shuffle scan, ballot compaction)
		int acc = 0, na = 0;
		for (int base = 0; base < NE; base += 32) {
			const int e = base + lane;
			const int c = e < NE ? cnt[e] : 0;
			int incl = c;
#pragma unroll
			for (int o = 1; o < 32; o <<= 1) {
				const int u = __shfl_up_sync(0xffffffffu, incl, o);
				if (lane >= o)
					incl += u;
			}
			const bool act = c > 0 && e >= first && e < first + nlocal;
			const unsigned m = __ballot_sync(0xffffffffu, act);
			if (e < NE) {
				offsets[e] = acc + incl - c;
				run[e] = acc + incl - c;
				counts[e] = c;
			}
			if (act)
				active[na + __popc(m & ((1u << lane) - 1u))] = e;
			na += __popc(m);
			acc += __shfl_sync(0xffffffffu, incl, 31);
		}
		if (lane == 0) {
			offsets[NE] = acc;
			*n_active = na;
		}
	}
	__syncthreads();

	for (int base = 0; base < npairs; base += blockDim.x) {
		for (int i = tid; i < nw * NE; i += blockDim.x)
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
			const int pos = run[e] + before + rank_w;
			perm[pos] = p;
			if (pos_of)
				pos_of[p] = pos;
		}
		__syncthreads();
		for (int e2 = tid; e2 < NE; e2 += blockDim.x) {
			int add = 0;
			for (int w = 0; w < nw; w++)
				add += wcnt[w * NE + e2];
			run[e2] += add;
		}
		__syncthreads();
	}
}

}  // namespace moe
