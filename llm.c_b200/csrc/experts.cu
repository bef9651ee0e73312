// experts.cu — grouped expert GEMV (decode path), combine, bias add.
//
// Reference: fused_ffn_fn (nn.c:449-493) computes, per (token, expert),
// gate/up rows with dot_f32_quant (quant.c:103-155), h = silu(g)*u, then
// the down rows over h; moe_ffn (olmoe.c:397-404) adds y / (1/w) into the
// token's output in top-k slot order.  Here the (token, slot) pairs are
// grouped by expert (dispatch in router.cu), each expert's weight rows are
// streamed once for all of its tokens, and the combine runs afterwards in
// slot order, so the output is deterministic.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace moe {

// ---------------------------------------------------------------------
// Simple grouped GEMV: one warp walks one weight row block by block; lane
// j owns element j of each 32-element block (lanes 0-15 take the low
// nibbles and 16-31 the high nibbles of a Q4_0 block).  Used for the
// single-expert drop-ins and as the cross-check of the tensor-core path.
// ---------------------------------------------------------------------
constexpr int kGemvTok = 8;        // tokens per pass (x tile in smem)
constexpr int kGemvWarps = 8;
constexpr int kGemvRowsPerWarp = 4;
constexpr int kGemvRows = kGemvWarps * kGemvRowsPerWarp;

template <int QT>
__device__ __forceinline__ float load_weight(const uint8_t *blk, int lane)
{
	const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk));
	if (QT == kQ8_0) {
		const float q = (float)(int8_t)blk[2 + lane];
		return __fmul_rn(d, q);
	} else {
		const uint8_t b = blk[2 + (lane & 15)];
		const int nib = lane < 16 ? (b & 15) : (b >> 4);
		return __fmul_rn(d, (float)(nib - 8));
	}
}

template <int QT, bool DUAL>
__global__ void __launch_bounds__(kGemvWarps * 32)
expert_gemv_kernel(GemvArgs a)
{
	extern __shared__ float xs[];  // [kGemvTok][cols]
	const int e = a.first_expert + blockIdx.x;
	const int n = a.counts[e];
	if (n == 0)
		return;
	const int off = a.offsets[e];
	const int cols = a.cols;
	const int64_t rb = row_bytes(QT, cols);
	const int bb = (int)block_bytes(QT);
	const int nblk = cols / QK;
	const uint8_t *W1 = static_cast<const uint8_t *>(a.w1[e]);
	const uint8_t *W2 = DUAL ? static_cast<const uint8_t *>(a.w2[e]) : nullptr;
	const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
	const int r0 = blockIdx.y * kGemvRows + warp * kGemvRowsPerWarp;

	for (int tb = 0; tb < n; tb += a.tok) {
		const int nt = min(a.tok, n - tb);
		__syncthreads();
		for (int i = threadIdx.x; i < nt * cols; i += blockDim.x) {
			const int tt = i / cols, k = i - tt * cols;
			const int pos = off + tb + tt;
			const int row = a.in_perm ? a.perm[pos] / a.K : pos;
			xs[i] = a.in[(int64_t)row * cols + k];
		}
		__syncthreads();
		for (int rr = 0; rr < kGemvRowsPerWarp; rr++) {
			const int r = r0 + rr;
			if (r >= a.rows)
				break;
			float acc1[kGemvTok], acc2[kGemvTok];
#pragma unroll
			for (int tt = 0; tt < kGemvTok; tt++)
				acc1[tt] = acc2[tt] = 0.0f;
			const uint8_t *p1 = W1 + (int64_t)r * rb;
			const uint8_t *p2 = DUAL ? W2 + (int64_t)r * rb : nullptr;
			for (int b = 0; b < nblk; b++) {
				const float w1 = load_weight<QT>(p1 + (int64_t)b * bb, lane);
				const float w2 = DUAL ? load_weight<QT>(p2 + (int64_t)b * bb, lane) : 0.0f;
				const float *xc = xs + b * QK + lane;
#pragma unroll
				for (int tt = 0; tt < kGemvTok; tt++) {
					if (tt < nt) {
						const float xv = xc[tt * cols];
						acc1[tt] = __fmaf_rn(w1, xv, acc1[tt]);
						if (DUAL)
							acc2[tt] = __fmaf_rn(w2, xv, acc2[tt]);
					}
				}
			}
#pragma unroll
			for (int tt = 0; tt < kGemvTok; tt++) {
				const float g = warp_sum(acc1[tt]);
				const float u = DUAL ? warp_sum(acc2[tt]) : 0.0f;
				if (lane == tt && tt < nt) {
					const int pos = off + tb + tt;
					const int orow = a.out_perm ? a.perm[pos] : pos;
					a.out[(int64_t)orow * a.rows + r] = DUAL ? swiglu(g, u) : g;
				}
			}
		}
	}
}

cudaError_t launch_expert_gemv(const GemvArgs &a, cudaStream_t st)
{
	if (a.n_local <= 0 || a.rows <= 0)
		return cudaSuccess;
	dim3 grid(a.n_local, (a.rows + kGemvRows - 1) / kGemvRows);
	// tokens per pass: as many as fit in ~200 KB of shared memory, at most 8
	GemvArgs b = a;
	b.tok = (int)std::min<int64_t>(kGemvTok, (200 * 1024) / ((int64_t)a.cols * 4));
	if (b.tok < 1)
		return cudaErrorInvalidValue;  // a row longer than 51200 elements
	size_t smem = (size_t)b.tok * a.cols * sizeof(float);
	void (*fn)(GemvArgs);
	if (a.qtype == kQ8_0)
		fn = a.dual ? expert_gemv_kernel<kQ8_0, true> : expert_gemv_kernel<kQ8_0, false>;
	else
		fn = a.dual ? expert_gemv_kernel<kQ4_0, true> : expert_gemv_kernel<kQ4_0, false>;
	cudaError_t e = ensure_smem(fn, smem);
	if (e != cudaSuccess)
		return e;
	fn<<<grid, kGemvWarps * 32, smem, st>>>(b);
	return cudaGetLastError();
}

// ---------------------------------------------------------------------
// combine: out[t] = ((0 + y0/(1/w0)) + y1/(1/w1)) + ...  (olmoe.c:397-404,
// tensor_div_scalar tensor.c:435-456 then tensor_add tensor.c:334-353)
// ---------------------------------------------------------------------
__global__ void combine_kernel(const float *__restrict__ Y, const float *__restrict__ w, int T,
			       int K, int d, float *__restrict__ out)
{
	// one thread per 4 consecutive outputs of one token (d % 4 == 0)
	const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
	const int d4 = d / 4;
	if (i >= (int64_t)T * d4)
		return;
	const int t = (int)(i / d4);
	const int j4 = (int)(i - (int64_t)t * d4);
	float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
	for (int s = 0; s < K; s++) {
		const float inv = __fdiv_rn(1.0f, w[t * K + s]);
		const float4 y = __ldg(reinterpret_cast<const float4 *>(Y + ((int64_t)t * K + s) * d) + j4);
		acc.x = __fadd_rn(__fdiv_rn(y.x, inv), acc.x);
		acc.y = __fadd_rn(__fdiv_rn(y.y, inv), acc.y);
		acc.z = __fadd_rn(__fdiv_rn(y.z, inv), acc.z);
		acc.w = __fadd_rn(__fdiv_rn(y.w, inv), acc.w);
	}
	reinterpret_cast<float4 *>(out + (int64_t)t * d)[j4] = acc;
}

__global__ void combine_kernel_scalar(const float *__restrict__ Y, const float *__restrict__ w,
				      int T, int K, int d, float *__restrict__ out)
{
	const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
	if (i >= (int64_t)T * d)
		return;
	const int t = (int)(i / d);
	const int j = (int)(i - (int64_t)t * d);
	float acc = 0.0f;
	for (int s = 0; s < K; s++) {
		const float inv = __fdiv_rn(1.0f, w[t * K + s]);
		const float y = __fdiv_rn(Y[((int64_t)t * K + s) * d + j], inv);
		acc = __fadd_rn(y, acc);
	}
	out[i] = acc;
}

cudaError_t launch_combine(const float *Y, const float *w, int T, int K, int d, float *out,
			   cudaStream_t st)
{
	const int64_t total = (int64_t)T * d;
	if (total == 0)
		return cudaSuccess;
	if (d % 4 == 0 && (uintptr_t)Y % 16 == 0 && (uintptr_t)out % 16 == 0) {
		const int64_t n4 = total / 4;
		combine_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(Y, w, T, K, d, out);
	} else {
		combine_kernel_scalar<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(Y, w, T, K, d,
											 out);
	}
	return cudaGetLastError();
}

// combine of rows stored at the pairs' dispatch positions (token-sharded
// expert parallelism): out[t] = sum_s Y[pos_of[t*K + s]] / (1 / w[t*K + s])
// in slot order, the same arithmetic as combine_kernel
__global__ void combine_pos_kernel(const float *__restrict__ Y, const int32_t *__restrict__ pos_of,
				   const float *__restrict__ w, int T, int K, int d,
				   float *__restrict__ out)
{
	const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
	const int d4 = d / 4;
	if (i >= (int64_t)T * d4)
		return;
	const int t = (int)(i / d4);
	const int j4 = (int)(i - (int64_t)t * d4);
	float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
	for (int s = 0; s < K; s++) {
		const float inv = __fdiv_rn(1.0f, w[t * K + s]);
		const int64_t row = pos_of[t * K + s];
		const float4 y = __ldg(reinterpret_cast<const float4 *>(Y + row * d) + j4);
		acc.x = __fadd_rn(__fdiv_rn(y.x, inv), acc.x);
		acc.y = __fadd_rn(__fdiv_rn(y.y, inv), acc.y);
		acc.z = __fadd_rn(__fdiv_rn(y.z, inv), acc.z);
		acc.w = __fadd_rn(__fdiv_rn(y.w, inv), acc.w);
	}
	reinterpret_cast<float4 *>(out + (int64_t)t * d)[j4] = acc;
}

cudaError_t launch_combine_pos(const float *Y, const int32_t *pos_of, const float *w, int T, int K,
			       int d, float *out, cudaStream_t st)
{
	const int64_t n4 = (int64_t)T * d / 4;
	if (n4 == 0)
		return cudaSuccess;
	if (d % 4 || (uintptr_t)Y % 16 || (uintptr_t)out % 16)
		return cudaErrorInvalidValue;
	combine_pos_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(Y, pos_of, w, T, K, d, out);
	return cudaGetLastError();
}

// rows moved by segment (token-sharded all-to-all): seg[i] = (source-major
// row, expert-major row, rows); dir 0 copies source-major -> expert-major,
// dir 1 the reverse.  blockIdx.y = segment, 16-byte chunks.
__global__ void copy_segments_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst,
				     const int64_t *__restrict__ seg, int dir, int64_t row_bytes)
{
	const int i = blockIdx.y;
	const int64_t from = seg[3 * i + (dir ? 1 : 0)], to = seg[3 * i + (dir ? 0 : 1)];
	const int64_t chunks = seg[3 * i + 2] * row_bytes / 16;
	const uint4 *s = reinterpret_cast<const uint4 *>(src + from * row_bytes);
	uint4 *d = reinterpret_cast<uint4 *>(dst + to * row_bytes);
	for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < chunks;
	     c += (int64_t)gridDim.x * blockDim.x)
		d[c] = s[c];
}

cudaError_t launch_copy_segments(const void *src, void *dst, const int64_t *seg, int nseg, int dir,
				 int64_t row_bytes, cudaStream_t st)
{
	if (nseg <= 0)
		return cudaSuccess;
	if (row_bytes % 16 || (uintptr_t)src % 16 || (uintptr_t)dst % 16 || nseg > 65535)
		return cudaErrorInvalidValue;
	copy_segments_kernel<<<dim3(32, (unsigned)nseg), 256, 0, st>>>(
		static_cast<const uint8_t *>(src), static_cast<uint8_t *>(dst), seg, dir, row_bytes);
	return cudaGetLastError();
}

__global__ void add_bias_kernel(float *ret, const float *add, int64_t total, int64_t n_add)
{
	const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
	if (i < total)
		ret[i] = __fadd_rn(add[i % n_add], ret[i]);
}

cudaError_t launch_add_bias(float *ret, const float *add, int64_t total, int64_t n_add,
			    cudaStream_t st)
{
	if (total == 0)
		return cudaSuccess;
	add_bias_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(ret, add, total, n_add);
	return cudaGetLastError();
}

}  // namespace moe
