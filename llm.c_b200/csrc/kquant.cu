// kquant.cu — MoE experts in the K-quant formats of the reference's real
// checkpoints (Q4_K, Q6_K; quant.h:30-57), for the decode-sized expert
// products: CUDA-core GEMVs, dequantization in registers, warp reductions.
//
// They compute what the reference's Q8_DOT build computes (nn.c:449-539):
//   gate/up: x quantized to Q8_K (quant.c:627-654), then per 256-block the
//            exact integer sum S (and, for Q4_K, the mins term M) of
//            quant_avx2.h, combined in block order as acc = fma(d, S, acc)
//            (acc_m likewise), result acc + acc_m — the same operations;
//   h = g / (1 + exp(-g)) * u;
//   down:    the fp32 dot of h with the dequantized row; element values as
//            quant.c:198-418 forms them ((d*sc)*q - dmin*m, (q-32)*(d*sc)),
//            summed over a warp instead of the reference's SIMD lanes (the
//            one place the order differs: fp32 rounding only).
//
// Expert segments follow the dispatch of route_core.cuh: the pairs of
// expert e are positions offsets[e] .. offsets[e] + counts[e] - 1 of perm.
#include "common.cuh"
#include "kernels.h"

namespace moe {

namespace {

constexpr int kKqWarps = 8;   // rows per CTA (one warp per row)

__device__ __forceinline__ uint32_t ldu32(const uint8_t *p)
{
	return *reinterpret_cast<const uint32_t *>(p);
}

__device__ __forceinline__ float f16_at(const uint8_t *p)
{
	return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// get_scale_min_k4 (quant.h:62-71)
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t *q, int &d, int &m)
{
	if (j < 4) {
		d = q[j] & 63;
		m = q[j + 4] & 63;
	} else {
		d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
		m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
	}
}

// ------------------------------------------------------------ Q8_K
// one CTA of 256 threads per (token, 256-block); y: [T][D/256] blocks of
// {float d; int8 qs[256]; int16 bsums[16]} (292 bytes)
__global__ void __launch_bounds__(256)
quantize_q8k_kernel(const float *__restrict__ x, int D, uint8_t *__restrict__ y)
{
	__shared__ float sa[8];
	__shared__ int si[8];
	const int t = blockIdx.y, b = blockIdx.x, j = threadIdx.x;
	const int nb = D / 256;
	const float v = x[(int64_t)t * D + b * 256 + j];
	// the first element of the largest magnitude (quant.c:633-636)
	float a = fabsf(v);
	int idx = j;
	for (int off = 16; off; off >>= 1) {
		const float oa = __shfl_xor_sync(0xffffffffu, a, off);
		const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
		if (oa > a || (oa == a && oi < idx)) {
			a = oa;
			idx = oi;
		}
	}
	if (j % 32 == 0) {
		sa[j / 32] = a;
		si[j / 32] = idx;
	}
	__syncthreads();
	if (j < 32) {
		a = j < 8 ? sa[j] : -1.0f;
		idx = j < 8 ? si[j] : 256;
		for (int off = 4; off; off >>= 1) {
			const float oa = __shfl_xor_sync(0xffffffffu, a, off);
			const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
			if (oa > a || (oa == a && oi < idx)) {
				a = oa;
				idx = oi;
			}
		}
		if (j == 0) {
			sa[0] = a;
			si[0] = idx;
		}
	}
	__syncthreads();
	const float amax = sa[0];
	uint8_t *blk = y + ((int64_t)t * nb + b) * 292;
	int q = 0;
	if (amax > 0.0f) {
		const float mval = x[(int64_t)t * D + b * 256 + si[0]];
		const float iscale = __fdiv_rn(-127.0f, mval);
		if (j == 0)
			*reinterpret_cast<float *>(blk) = __fdiv_rn(1.0f, iscale);
		const int r = (int)roundf(__fmul_rn(iscale, v));
		q = r < 127 ? r : 127;
	} else if (j == 0) {
		*reinterpret_cast<float *>(blk) = 0.0f;
	}
	blk[4 + j] = (uint8_t)(int8_t)q;
	// bsums: the 16 values of each half-warp
	int s = q;
	for (int off = 8; off; off >>= 1)
		s += __shfl_xor_sync(0xffffffffu, s, off);
	if (j % 16 == 0)
		reinterpret_cast<int16_t *>(blk + 260)[j / 16] = (int16_t)s;
}

// ------------------------------------------------------------ gate / up
// One 256-block of a Q4_K row against one Q8_K block, by a warp: lane l
// takes code bytes 4l..4l+3 (elements 64j + 4(l%8) .. +3 of sub-block 2j,
// their high nibbles those of sub-block 2j + 1, j = l / 8).  S and M are
// exact, so the warp's order is the reference's.
__device__ __forceinline__ void q4k_block(const uint8_t *wb, const uint8_t *yb, int lane, int &S,
					  int &M)
{
	const int j = lane >> 3, k = 4 * (lane & 7);
	const uint8_t *sc = wb + 4;
	int s_lo, m_lo, s_hi, m_hi;
	scale_min_k4(2 * j, sc, s_lo, m_lo);
	scale_min_k4(2 * j + 1, sc, s_hi, m_hi);
	const uint32_t w = ldu32(wb + 16 + 4 * lane);
	const int lo = __dp4a((int)(w & 0x0F0F0F0Fu), (int)ldu32(yb + 4 + 64 * j + k), 0);
	const int hi = __dp4a((int)((w >> 4) & 0x0F0F0F0Fu), (int)ldu32(yb + 4 + 64 * j + 32 + k), 0);
	S = s_lo * lo + s_hi * hi;
	// the mins term: lane s < 8 takes sub-block s
	M = 0;
	if (lane < 8) {
		int sd, m;
		scale_min_k4(lane, sc, sd, m);
		const int16_t *bs = reinterpret_cast<const int16_t *>(yb + 260);
		M = m * ((int)bs[2 * lane] + (int)bs[2 * lane + 1]);
	}
}

// Q6_K: lane l takes element l of each of the 8 groups of 32 (two halves
// of 128, four groups each); value (6 bits) - 32, scale per 16 elements
__device__ __forceinline__ int q6k_block(const uint8_t *wb, const uint8_t *yb, int lane)
{
	const int8_t *qs = reinterpret_cast<const int8_t *>(yb + 4);
	const int8_t *scales = reinterpret_cast<const int8_t *>(wb + 192);
	int S = 0;
#pragma unroll
	for (int h = 0; h < 2; h++) {
		const int a = wb[h * 64 + lane], c = wb[h * 64 + 32 + lane], hb = wb[128 + h * 32 + lane];
		const int q0 = ((a & 15) | ((hb & 3) << 4)) - 32;
		const int q1 = ((c & 15) | (((hb >> 2) & 3) << 4)) - 32;
		const int q2 = ((a >> 4) | (((hb >> 4) & 3) << 4)) - 32;
		const int q3 = ((c >> 4) | (((hb >> 6) & 3) << 4)) - 32;
		const int e = h * 128 + lane, hi16 = lane >= 16;
		S += scales[h * 8 + 0 + hi16] * q0 * qs[e];
		S += scales[h * 8 + 2 + hi16] * q1 * qs[e + 32];
		S += scales[h * 8 + 4 + hi16] * q2 * qs[e + 64];
		S += scales[h * 8 + 6 + hi16] * q3 * qs[e + 96];
	}
	return S;
}

__device__ __forceinline__ int warp_isum(int v)
{
	for (int off = 16; off; off >>= 1)
		v += __shfl_xor_sync(0xffffffffu, v, off);
	return v;
}

// row `row` (nb blocks of type QT) against token q8k row yt: the
// reference's dot_q8_quant result, in lane 0
template <int QT>
__device__ float kq_dot_q8k(const uint8_t *row, const uint8_t *yt, int nb, int lane)
{
	float acc = 0.0f, acc_m = 0.0f;
	for (int b = 0; b < nb; b++) {
		const uint8_t *yb = yt + b * 292;
		const float d8 = *reinterpret_cast<const float *>(yb);
		if (QT == kQ4_K) {
			const uint8_t *wb = row + b * 144;
			int S, M;
			q4k_block(wb, yb, lane, S, M);
			S = warp_isum(S);
			M = warp_isum(M);
			const float d = __fmul_rn(d8, f16_at(wb));
			const float dmin = __fmul_rn(-d8, f16_at(wb + 2));
			acc_m = __fmaf_rn(dmin, (float)M, acc_m);
			acc = __fmaf_rn(d, (float)S, acc);
		} else {
			const uint8_t *wb = row + b * 210;
			const int S = warp_isum(q6k_block(wb, yb, lane));
			const float d = __fmul_rn(d8, f16_at(wb + 208));
			acc = __fmaf_rn(d, (float)S, acc);
		}
	}
	return __fadd_rn(acc, acc_m);
}

}  // namespace

namespace {

// grid (row groups of kKqWarps rows, local experts): warp w of CTA (g, e)
// takes row g * kKqWarps + w of expert first + e for every pair of the
// expert's segment: h[pos][row] = swiglu(gate . x8, up . x8)
template <int QT>
__global__ void __launch_bounds__(kKqWarps * 32) kq_gate_up_kernel(KqArgs a)
{
	const int e = a.first_expert + blockIdx.y;
	const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
	const int row = blockIdx.x * kKqWarps + warp;
	const int n = a.counts[e];
	if (n == 0 || row >= a.rows)
		return;
	const int nb = a.cols / 256;
	const int64_t rb = (int64_t)nb * (QT == kQ4_K ? 144 : 210);
	const uint8_t *g = static_cast<const uint8_t *>(a.w1[e]) + row * rb;
	const uint8_t *u = static_cast<const uint8_t *>(a.w2[e]) + row * rb;
	const int off = a.offsets[e];
	for (int i = 0; i < n; i++) {
		const int pos = off + i;
		const int t = a.perm[pos] / a.K;
		const uint8_t *yt = a.x8 + (int64_t)t * nb * 292;
		const float gv = kq_dot_q8k<QT>(g, yt, nb, lane);
		const float uv = kq_dot_q8k<QT>(u, yt, nb, lane);
		if (lane == 0)
			a.h[(int64_t)pos * a.rows + row] = swiglu(gv, uv);
	}
}

// down: Y[perm[pos]][row] = h[pos] . row (fp32 dot of the dequantized row)
template <int QT>
__global__ void __launch_bounds__(kKqWarps * 32) kq_down_kernel(KqArgs a)
{
	const int e = a.first_expert + blockIdx.y;
	const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
	const int row = blockIdx.x * kKqWarps + warp;
	const int n = a.counts[e];
	if (n == 0 || row >= a.rows)
		return;
	const int nb = a.cols / 256;
	const int64_t rb = (int64_t)nb * (QT == kQ4_K ? 144 : 210);
	const uint8_t *w = static_cast<const uint8_t *>(a.w1[e]) + row * rb;
	const int off = a.offsets[e];
	for (int i = 0; i < n; i++) {
		const int pos = off + i;
		const float *hp = a.hin + (int64_t)pos * a.cols;
		float acc = 0.0f;
		for (int b = 0; b < nb; b++) {
			const float *hb = hp + b * 256;
			if (QT == kQ4_K) {
				// quant.c:200-236: value (d*sc)*q - dmin*m, products rounded
				const uint8_t *wb = w + b * 144;
				const float d = f16_at(wb), dmin = f16_at(wb + 2);
				const int j = lane >> 3, k = 4 * (lane & 7);
				int s1, m1, s2, m2;
				scale_min_k4(2 * j, wb + 4, s1, m1);
				scale_min_k4(2 * j + 1, wb + 4, s2, m2);
				const float d1 = __fmul_rn(d, (float)s1), n1 = __fmul_rn(dmin, (float)m1);
				const float d2 = __fmul_rn(d, (float)s2), n2 = __fmul_rn(dmin, (float)m2);
				const uint32_t q = ldu32(wb + 16 + 4 * lane);
				const float4 xl = *reinterpret_cast<const float4 *>(hb + 64 * j + k);
				const float4 xh = *reinterpret_cast<const float4 *>(hb + 64 * j + 32 + k);
				const float xlv[4] = {xl.x, xl.y, xl.z, xl.w}, xhv[4] = {xh.x, xh.y, xh.z, xh.w};
#pragma unroll
				for (int c = 0; c < 4; c++) {
					const int byte = (q >> (8 * c)) & 0xFF;
					acc = __fmaf_rn(__fsub_rn(__fmul_rn(d1, (float)(byte & 15)), n1), xlv[c], acc);
					acc = __fmaf_rn(__fsub_rn(__fmul_rn(d2, (float)(byte >> 4)), n2), xhv[c], acc);
				}
			} else {
				// quant.c:305-410: value (float)(q - 32) * (d * scale)
				const uint8_t *wb = w + b * 210;
				const float d = f16_at(wb + 208);
				const int8_t *scales = reinterpret_cast<const int8_t *>(wb + 192);
#pragma unroll
				for (int h = 0; h < 2; h++) {
					const int qa = wb[h * 64 + lane], qc = wb[h * 64 + 32 + lane];
					const int hb2 = wb[128 + h * 32 + lane], hi16 = lane >= 16;
					const int qv[4] = {((qa & 15) | ((hb2 & 3) << 4)) - 32,
							   ((qc & 15) | (((hb2 >> 2) & 3) << 4)) - 32,
							   ((qa >> 4) | (((hb2 >> 4) & 3) << 4)) - 32,
							   ((qc >> 4) | (((hb2 >> 6) & 3) << 4)) - 32};
#pragma unroll
					for (int g = 0; g < 4; g++) {
						const float vs = __fmul_rn(d, (float)scales[h * 8 + 2 * g + hi16]);
						acc = __fmaf_rn(__fmul_rn((float)qv[g], vs),
								hb[h * 128 + 32 * g + lane], acc);
					}
				}
			}
		}
		acc = warp_sum(acc);
		if (lane == 0)
			a.out[(int64_t)a.perm[pos] * a.rows + row] = acc;
	}
}

}  // namespace

bool kquant_type(int qtype) { return qtype == kQ4_K || qtype == kQ6_K; }

cudaError_t launch_quantize_q8k(const float *x, int T, int D, uint8_t *y, cudaStream_t st)
{
	if (T <= 0)
		return cudaSuccess;
	if (D % 256)
		return cudaErrorInvalidValue;
	quantize_q8k_kernel<<<dim3(D / 256, T), 256, 0, st>>>(x, D, y);
	return cudaGetLastError();
}

cudaError_t launch_kq_gate_up(const KqArgs &a, int qtype, cudaStream_t st)
{
	if (a.cols % 256 || a.n_local <= 0)
		return cudaErrorInvalidValue;
	const dim3 grid((a.rows + kKqWarps - 1) / kKqWarps, a.n_local);
	if (qtype == kQ4_K)
		kq_gate_up_kernel<kQ4_K><<<grid, kKqWarps * 32, 0, st>>>(a);
	else if (qtype == kQ6_K)
		kq_gate_up_kernel<kQ6_K><<<grid, kKqWarps * 32, 0, st>>>(a);
	else
		return cudaErrorInvalidValue;
	return cudaGetLastError();
}

cudaError_t launch_kq_down(const KqArgs &a, int qtype, cudaStream_t st)
{
	if (a.cols % 256 || a.n_local <= 0)
		return cudaErrorInvalidValue;
	const dim3 grid((a.rows + kKqWarps - 1) / kKqWarps, a.n_local);
	if (qtype == kQ4_K)
		kq_down_kernel<kQ4_K><<<grid, kKqWarps * 32, 0, st>>>(a);
	else if (qtype == kQ6_K)
		kq_down_kernel<kQ6_K><<<grid, kKqWarps * 32, 0, st>>>(a);
	else
		return cudaErrorInvalidValue;
	return cudaGetLastError();
}

}  // namespace moe
