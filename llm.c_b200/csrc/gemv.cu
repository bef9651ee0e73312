// gemv.cu — the single-token quantized GEMV y = W x: config 1's dense
// decode shape (W 14336 x 4096 Q4_0, x 1 x 4096), and the dense drop-in when
// the caller passes one activation row (matmul.c:291-305 -> 107-131).
//
// Memory-bound, so no tensor cores and no staging: one warp per weight row,
// lane l reading blocks l, l + 32, ... of it (a warp's loads cover 32
// consecutive blocks, 576 / 1088 contiguous bytes), dequantized in registers
// and multiplied with x from shared memory in fp32.
//
// * Blocks are 18 / 34 bytes, so a block starts 0 or 2 bytes past a 4-byte
//   boundary: each lane reads the 5 / 9 aligned words from the boundary at
//   or below its block, and funnel shifts take the codes out of them.  With
//   an even number of blocks per row (cols % 64 == 0) those words never
//   reach past the row, or past the matrix for its last row.
// * A code becomes an exact fp32 value without an int-to-float conversion
//   (a quarter-rate instruction): one byte permute writes code + 128 (Q8_0)
//   or the nibble (Q4_0) into the mantissa of 2^23, one subtraction removes
//   2^23 and the offset.  Products and the block's 32-term sum are fp32; the
//   block's fp16 scale multiplies the sum, as dot_f32_quant does per block.
//   The sums are not in the reference's SIMD-lane order, so the result
//   agrees with it to fp32 rounding (~1e-7 relative), not bit for bit.
// * x is held in shared memory 36 floats per block (32 + 4 of padding), so
//   the float4 reads of the 32 lanes (32 different blocks) spread over all
//   banks.
#include "common.cuh"
#include "kernels.h"

namespace moe {

namespace {

constexpr int kG1Threads = 256;
constexpr int kXPad = 36;   // floats per block of x in shared memory
constexpr int kBL = 4;      // blocks a lane loads before converting them
constexpr int kG1MinBlocks = 8;  // 8 CTAs (64 warps) per SM: at most 32 registers

// the float 2^23 + (byte j of w): the permute puts the byte in the low
// mantissa bits and 0x4B (the exponent of 2^23) in the top byte
__device__ __forceinline__ float byte_as_f(uint32_t w, int j)
{
	return __int_as_float((int)__byte_perm(w, 0x4B000000u, 0x7540u | (uint32_t)j));
}

template <int QT>
__global__ void __launch_bounds__(kG1Threads, kG1MinBlocks)
gemv1_kernel(const uint8_t *__restrict__ w, int rows, int nb, const float *__restrict__ x,
	     float *__restrict__ y)
{
	constexpr int BB = QT == kQ8_0 ? Q8_0_BYTES : Q4_0_BYTES;
	constexpr int NW = BB / 4 + 1;   // aligned words that cover a block (9 / 5)
	constexpr int NC = QT == kQ8_0 ? 8 : 4;  // code words of a block
	extern __shared__ __align__(16) float xs[];   // [nb][kXPad]
	for (int i = threadIdx.x; i < nb * 8; i += blockDim.x)
		reinterpret_cast<float4 *>(xs + (i >> 3) * kXPad)[i & 7] =
			__ldg(reinterpret_cast<const float4 *>(x) + i);
	__syncthreads();
	const int lane = threadIdx.x & 31;
	const int64_t rb = (int64_t)nb * BB;
	const int nwarps = gridDim.x * (blockDim.x / 32);
	for (int r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < rows; r += nwarps) {
		const uint8_t *row = w + (int64_t)r * rb;
		float acc = 0.0f;
		// kBL blocks per lane per round: all their words are loaded first
		for (int b0 = lane; b0 < nb; b0 += 32 * kBL) {
			uint32_t v[kBL][NW];
#pragma unroll
			for (int u = 0; u < kBL; u++) {
				const int b = b0 + 32 * u < nb ? b0 + 32 * u : b0;
				const uint32_t *p = reinterpret_cast<const uint32_t *>(
					reinterpret_cast<uintptr_t>(row + (int64_t)b * BB) & ~uintptr_t(3));
#pragma unroll
				for (int k = 0; k < NW; k++)
					v[u][k] = __ldg(p + k);
			}
#pragma unroll
			for (int u = 0; u < kBL; u++) {
				const int b = b0 + 32 * u;
				// block 2 bytes past a 4-byte boundary (odd block of the row)
				const bool odd = (b & 1) != 0;
				// scale: block bytes 0-1; codes: block bytes 2.. = window bytes
				// 2.. (aligned block) or 4.. (block 2 bytes past the boundary)
				const float d = __half2float(__ushort_as_half(
					(unsigned short)((odd ? v[u][0] >> 16 : v[u][0]) & 0xFFFFu)));
				uint32_t c[NC];
#pragma unroll
				for (int k = 0; k < NC; k++)
					c[k] = odd ? v[u][k + 1] : __funnelshift_r(v[u][k], v[u][k + 1], 16);
				const float *xb = xs + (b < nb ? b : b0) * kXPad;
				float s = 0.0f;
				if (QT == kQ8_0) {
					// code j (int8) at byte j: byte ^ 0x80 = q + 128
#pragma unroll
					for (int k = 0; k < 8; k++) {
						const uint32_t q = c[k] ^ 0x80808080u;
						const float4 xv = *reinterpret_cast<const float4 *>(xb + 4 * k);
						s = __fmaf_rn(byte_as_f(q, 0) - 8388736.0f, xv.x, s);
						s = __fmaf_rn(byte_as_f(q, 1) - 8388736.0f, xv.y, s);
						s = __fmaf_rn(byte_as_f(q, 2) - 8388736.0f, xv.z, s);
						s = __fmaf_rn(byte_as_f(q, 3) - 8388736.0f, xv.w, s);
					}
				} else {
					// byte j: element j in its low nibble, element j + 16 in
					// its high nibble; values nib - 8
#pragma unroll
					for (int k = 0; k < 4; k++) {
						const uint32_t lo = c[k] & 0x0F0F0F0Fu, hi = (c[k] >> 4) & 0x0F0F0F0Fu;
						const float4 xl = *reinterpret_cast<const float4 *>(xb + 4 * k);
						const float4 xh = *reinterpret_cast<const float4 *>(xb + 16 + 4 * k);
						s = __fmaf_rn(byte_as_f(lo, 0) - 8388616.0f, xl.x, s);
						s = __fmaf_rn(byte_as_f(lo, 1) - 8388616.0f, xl.y, s);
						s = __fmaf_rn(byte_as_f(lo, 2) - 8388616.0f, xl.z, s);
						s = __fmaf_rn(byte_as_f(lo, 3) - 8388616.0f, xl.w, s);
						s = __fmaf_rn(byte_as_f(hi, 0) - 8388616.0f, xh.x, s);
						s = __fmaf_rn(byte_as_f(hi, 1) - 8388616.0f, xh.y, s);
						s = __fmaf_rn(byte_as_f(hi, 2) - 8388616.0f, xh.z, s);
						s = __fmaf_rn(byte_as_f(hi, 3) - 8388616.0f, xh.w, s);
					}
				}
				if (b < nb)
					acc = __fmaf_rn(d, s, acc);
			}
		}
#pragma unroll
		for (int o = 16; o >= 1; o >>= 1)
			acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
		if (lane == 0)
			y[r] = acc;
	}
}

}  // namespace

bool gemv1_supported(int qtype, int64_t rows, int64_t cols, uintptr_t w, uintptr_t x, uintptr_t y)
{
	return (qtype == kQ8_0 || qtype == kQ4_0) && rows > 0 && rows <= INT32_MAX && cols > 0 &&
	       cols % 64 == 0 && cols / QK * kXPad * 4 <= 200 * 1024 && w % 4 == 0 && x % 16 == 0 &&
	       y % 4 == 0;
}

cudaError_t launch_gemv1(const void *w, int qtype, int64_t rows, int64_t cols, const float *x,
			 float *y, cudaStream_t st)
{
	const int nb = (int)(cols / QK);
	const size_t smem = (size_t)nb * kXPad * 4;
	int64_t grid = (rows + kG1Threads / 32 - 1) / (kG1Threads / 32);
	if (grid > (int64_t)sm_count() * 8)
		grid = (int64_t)sm_count() * 8;
	if (qtype == kQ8_0) {
		cudaError_t e = ensure_smem(gemv1_kernel<kQ8_0>, smem);
		if (e != cudaSuccess)
			return e;
		gemv1_kernel<kQ8_0><<<(unsigned)grid, kG1Threads, smem, st>>>(
			static_cast<const uint8_t *>(w), (int)rows, nb, x, y);
	} else {
		cudaError_t e = ensure_smem(gemv1_kernel<kQ4_0>, smem);
		if (e != cudaSuccess)
			return e;
		gemv1_kernel<kQ4_0><<<(unsigned)grid, kG1Threads, smem, st>>>(
			static_cast<const uint8_t *>(w), (int)rows, nb, x, y);
	}
	return cudaGetLastError();
}

}  // namespace moe
