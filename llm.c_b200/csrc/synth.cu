// synth.cu — seeded synthetic inputs and Q8_0/Q4_0 quantization on the
// device, for benches and tests that need full-size layers quickly.
//
// Generator: splitmix64 in counter form (draw n of stream s is
// mix64(s + n * 0x9E3779B97F4A7C15)), two draws per value through
// Box-Muller in double precision.  Quantizers follow the reference's
// rounding rules: Q8_0 as quantize_row_q8_0 (quant.c:62-78: d = amax/127
// stored as fp16 round-to-nearest-even, codes roundf(x * (1/d))); Q4_0 as
// the reference's only Q4_0 quantizer, in its tests (test/quant.c:45-79:
// d = amax/7 stored as fp16 by truncation, codes roundf(x * 7/amax) + 8
// clamped to 0..15, element j in the low nibble of byte j and element
// j+16 in its high nibble).
#include "common.cuh"
#include "kernels.h"

namespace moe {

__device__ __forceinline__ uint64_t mix64(uint64_t z)
{
	z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
	z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
	return z ^ (z >> 31);
}

__device__ __forceinline__ double unit_draw(uint64_t stream, uint64_t n)
{
	const uint64_t z = mix64(stream + n * 0x9E3779B97F4A7C15ULL);
	return ((double)(z >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

__global__ void synth_gauss_kernel(float *dst, uint64_t stream, uint64_t offset, int64_t n,
				   float sd)
{
	for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
	     i += (int64_t)gridDim.x * blockDim.x) {
		const uint64_t e = offset + (uint64_t)i;
		const double u1 = unit_draw(stream, 2 * e + 1);
		const double u2 = unit_draw(stream, 2 * e + 2);
		const double g = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
		dst[i] = (float)((double)sd * g);
	}
}

cudaError_t launch_synth_gauss(float *dst, uint64_t stream_seed, uint64_t offset, int64_t n,
			       float sd, cudaStream_t st)
{
	if (n <= 0)
		return cudaSuccess;
	int64_t blocks = (n + 255) / 256;
	if (blocks > 148 * 64)
		blocks = 148 * 64;
	synth_gauss_kernel<<<(unsigned)blocks, 256, 0, st>>>(dst, stream_seed, offset, n, sd);
	return cudaGetLastError();
}

// test/quant.c:19-33 truncating fp32 -> fp16
__device__ __forceinline__ uint16_t f16_trunc(float f)
{
	const uint32_t x = __float_as_uint(f);
	const uint32_t sign = (x >> 16) & 0x8000u;
	const uint32_t exp = (x >> 23) & 0xffu;
	const uint32_t man = x & 0x7fffffu;
	if (exp == 0)
		return (uint16_t)sign;
	if (exp == 0xff)
		return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
	const int e16 = (int)exp - 112;
	if (e16 >= 0x1f)
		return (uint16_t)(sign | 0x7c00u);
	if (e16 <= 0)
		return (uint16_t)sign;
	return (uint16_t)(sign | ((uint32_t)e16 << 10) | (man >> 13));
}

// fp32 -> fp16 bits, round to nearest even (the rounding of the
// reference's f32_to_f16, quant.c:46-60, and of F16C's _cvtss_sh), in
// integer arithmetic: normal halves round the 13 dropped mantissa bits,
// subnormal halves shift the full significand
__device__ __forceinline__ uint16_t f16_rne(float f)
{
	const uint32_t x = __float_as_uint(f);
	const uint32_t sign = (x >> 16) & 0x8000u;
	const uint32_t ax = x & 0x7fffffffu;
	if (ax > 0x7f800000u)
		return (uint16_t)(sign | 0x7e00u | ((ax >> 13) & 0x3ffu));
	if (ax >= 0x477ff000u)
		return (uint16_t)(sign | 0x7c00u);
	if (ax >= 0x38800000u) {
		uint32_t r = ax - 0x38000000u;
		r += 0x0fffu + ((r >> 13) & 1u);
		return (uint16_t)(sign | (r >> 13));
	}
	const uint32_t e = ax >> 23;
	if (e < 102)
		return (uint16_t)sign;
	const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
	const uint32_t sh = 126 - e;
	uint32_t q = m >> sh;
	const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
	if (rem > half || (rem == half && (q & 1u)))
		q++;
	return (uint16_t)(sign | q);
}

// one thread per 32-element block
__global__ void quantize_kernel(const float *__restrict__ src, int64_t nblocks, int qtype,
				uint8_t *__restrict__ dst)
{
	for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks;
	     b += (int64_t)gridDim.x * blockDim.x) {
		const float *x = src + b * QK;
		float amax = 0.0f;
		for (int j = 0; j < QK; j++) {
			const float a = fabsf(x[j]);
			if (a > amax)
				amax = a;
		}
		if (qtype == kQ8_0) {
			uint8_t *o = dst + b * Q8_0_BYTES;
			const float d = __fdiv_rn(amax, 127.0f);
			const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
			const uint16_t h = f16_rne(d);
			o[0] = (uint8_t)(h & 0xff);
			o[1] = (uint8_t)(h >> 8);
			for (int j = 0; j < QK; j++)
				o[2 + j] = (uint8_t)(int8_t)roundf(__fmul_rn(x[j], id));
		} else {
			uint8_t *o = dst + b * Q4_0_BYTES;
			const float scale = __fdiv_rn(amax, 7.0f);
			const float inv = scale > 0.0f ? __fdiv_rn(7.0f, amax) : 0.0f;
			const uint16_t h = f16_trunc(scale);
			o[0] = (uint8_t)(h & 0xff);
			o[1] = (uint8_t)(h >> 8);
			for (int j = 0; j < QK / 2; j++) {
				int lo = (int)roundf(__fmul_rn(x[j], inv)) + 8;
				int hi = (int)roundf(__fmul_rn(x[j + QK / 2], inv)) + 8;
				lo = lo < 0 ? 0 : (lo > 15 ? 15 : lo);
				hi = hi < 0 ? 0 : (hi > 15 ? 15 : hi);
				o[2 + j] = (uint8_t)(lo | (hi << 4));
			}
		}
	}
}

cudaError_t launch_quantize(const float *src, int64_t rows, int64_t cols, int qtype, void *dst,
			    cudaStream_t st)
{
	const int64_t nblocks = rows * (cols / QK);
	if (nblocks <= 0)
		return cudaSuccess;
	int64_t blocks = (nblocks + 255) / 256;
	if (blocks > 148 * 64)
		blocks = 148 * 64;
	quantize_kernel<<<(unsigned)blocks, 256, 0, st>>>(src, nblocks, qtype,
							   static_cast<uint8_t *>(dst));
	return cudaGetLastError();
}

}  // namespace moe
