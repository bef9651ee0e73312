// gemv.cu — the single-token quantized GEMV y = W x: config 1's dense
// decode shape (W 14336 x 4096 Q4_0, x 1 x 4096), and the dense drop-in when
// the caller passes one activation row (matmul.c:291-305 -> 107-131).
//
// gemv_tc_kernel (the default): a memory-bound stream of weight rows that
// must not stall on the math, and math that must stay well under the
// stream's time.
//
// * Streaming.  One CTA per SM owns a contiguous, row-balanced range of
//   rows (rows / SMs, not whole tiles).  A copy warp moves 16-row tiles
//   into a ring of 2-4 shared memory stages, one cp.async.bulk (the TMA
//   engine) per whole GGUF row, issued by 16 lanes at once, signalled by an
//   mbarrier; the math warps free a stage by arriving on its "empty"
//   mbarrier.  Every wait is bounded.  Rows sit 16 bytes apart beyond their
//   length in a stage: GGUF rows of 4096 (Q4_0) or 2048 (Q8_0) columns are
//   multiples of 128 bytes, so unpadded, the eight rows an MMA fragment
//   load touches would all fall in the same shared-memory bank.
// * Math.  The codes stay integers: an int8 tensor-core MMA
//   (mma.sync m16n8k32, codes as the 16 x 32 A tile straight from the
//   stage: Q8_0 as s8, Q4_0 nibbles as u8) multiplies them with x held as
//   three int8 digit planes per 32-element block: x = s (d1 + d2/254 +
//   d3/254^2) with s = amax/127, the planes being the MMA's n columns.
//   Each block's integer sums are exact; they become fp32 with the block's
//   fp16 weight scale and the plane scales (and, for Q4_0, minus 8 times the
//   plane's digit sum, the nibble bias).  The three planes carry x to ~2^-17
//   of the block maximum, so the result is within ~1e-6 relative of the
//   reference's fp32 arithmetic (dot_f32_q4_0 / dot_f32_q8_0, quant.c:103-155,
//   which multiplies dequantized weights by fp32 x).  About 37 instructions
//   per 16 rows x 32 codes instead of ~3 per code with fp32 FMAs, so the
//   math of a tile takes a fraction of the time its copy does.
// * The 8 math warps split each tile's blocks (K) eight ways; partial row
//   sums meet in shared memory and are added in warp order.
// * Every CTA splits x into digits itself (16 KB of x, from L2), while the
//   first copies are in flight.
//
// gemv1_kernel (shapes the ring does not fit): one warp per weight row, lane
// l reading blocks l, l + 32, ... with aligned 32-bit loads, codes made exact
// fp32 by a byte permute into 2^23, fp32 FMAs with x from shared memory.
#include "common.cuh"
#include "expert_core.cuh"
#include "kernels.h"

namespace moe {

namespace {

// ---------------------------------------------------------------- gemv_tc
constexpr int kTcMath = 8;                      // math warps
constexpr int kTcThreads = (kTcMath + 1) * 32;  // + the copy warp
constexpr int kTcRows = 16;                     // rows per tile (the MMA's M)
constexpr int kTcPlanes = 3;                    // int8 digit planes of x
constexpr int kTcMaxStages = 4;
constexpr size_t kTcSmemCap = 210 * 1024;

// shared memory after the stage ring, per block of x: digits [3][32] int8,
// plane scales [4] f32, plane digit sums [4] i32; then 32 zero bytes, the
// partial sums [2][kTcMath][16] f32 and the mbarriers
constexpr int kTcXd = kTcPlanes * 32, kTcPerBlock = kTcXd + 16 + 16;
// bytes between rows in a stage (conflict-free fragment loads)
__host__ __device__ inline int64_t tc_row_stride(int64_t rb) { return rb + 16; }
inline size_t tc_smem(int stages, int64_t tile_bytes, int nb)
{
	return (size_t)stages * tile_bytes + (size_t)nb * kTcPerBlock + 32 +
	       2 * kTcMath * kTcRows * 4 + 2 * kTcMaxStages * 8;
}

__device__ __forceinline__ void imma_16832(int32_t (&d)[4], const uint32_t (&a)[4], uint32_t b0,
					   uint32_t b1, bool a_unsigned)
{
	if (a_unsigned)
		asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
			     "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
			     : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
			     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
	else
		asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
			     "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
			     : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
			     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// 4 bytes at p, which lies 0 or 2 bytes past a 4-byte boundary
__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t *p)
{
	const uintptr_t a = reinterpret_cast<uintptr_t>(p);
	const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
	return (a & 2) ? __funnelshift_r(w[0], w[1], 16) : w[0];
}

template <int QT>
__global__ void __launch_bounds__(kTcThreads, 1)
gemv_tc_kernel(const uint8_t *__restrict__ w, int rows, int nb, int stages,
	       const float *__restrict__ x, float *__restrict__ y, int32_t *err)
{
	constexpr int BB = QT == kQ8_0 ? Q8_0_BYTES : Q4_0_BYTES;
	extern __shared__ __align__(128) uint8_t smem[];
	const int64_t rb = (int64_t)nb * BB;          // row bytes (a multiple of 16)
	const int64_t rs = tc_row_stride(rb);         // row stride in a stage
	const int64_t tile_bytes = kTcRows * rs;
	uint8_t *ring = smem;
	uint8_t *xd = smem + stages * tile_bytes;     // [nb][3][32] int8
	float *pw = reinterpret_cast<float *>(xd + (size_t)nb * kTcXd);  // [nb][4]
	int32_t *psum = reinterpret_cast<int32_t *>(pw + (size_t)nb * 4);  // [nb][4]
	uint8_t *zero = reinterpret_cast<uint8_t *>(psum + (size_t)nb * 4);  // 32 bytes
	float *red = reinterpret_cast<float *>(zero + 32);  // [2][kTcMath][16]
	uint64_t *full = reinterpret_cast<uint64_t *>(red + 2 * kTcMath * kTcRows);
	uint64_t *empty = full + kTcMaxStages;

	const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
	const int r0 = (int)((int64_t)blockIdx.x * rows / gridDim.x);
	const int r1 = (int)((int64_t)(blockIdx.x + 1) * rows / gridDim.x);
	const int ntiles = (r1 - r0 + kTcRows - 1) / kTcRows;
	if (tid == 0) {
		for (int i = 0; i < stages; i++) {
			mbar_init(&full[i], 1);
			mbar_init(&empty[i], kTcMath);
		}
		fence_mbar_init();
	}
	if (tid < 8)
		reinterpret_cast<uint32_t *>(zero)[tid] = 0;
	__syncthreads();

	if (warp == kTcMath) {
		// ---- copy warp: the rows of a tile, lane j copying row j
		bool failed = false;
		for (int i = 0; i < ntiles; i++) {
			const int slot = i % stages;
			if (i >= stages && !failed &&
			    !__all_sync(0xffffffffu, mbar_wait(&empty[slot], ((i / stages) - 1) & 1))) {
				failed = true;
				if (lane == 0 && err)
					atomicExch(err, 2);
			}
			if (failed)
				break;
			const int r = r0 + i * kTcRows;
			const int n = min(kTcRows, r1 - r);
			if (lane == 0)
				mbar_arrive_expect_tx(&full[slot], (uint32_t)(n * rb));
			__syncwarp();
			if (lane < n) {
				fence_proxy_async();
				bulk_g2s(ring + slot * tile_bytes + lane * rs, w + (int64_t)(r + lane) * rb,
					 (uint32_t)rb, &full[slot]);
			}
		}
		// no copy may still be landing when the CTA ends: wait for the last
		// `stages` copies (bounded)
		if (lane == 0)
			for (int i = max(0, ntiles - stages); i < ntiles && !failed; i++)
				if (!mbar_wait(&full[i % stages], (i / stages) & 1)) {
					failed = true;
					if (err)
						atomicExch(err, 2);
				}
		return;
	}

	// ---- math warps: x as three int8 digit planes per block (warp w takes
	// blocks w, w + 8, ...; lane k = element k of the block)
	for (int b = warp; b < nb; b += kTcMath) {
		const float v = __ldg(x + (int64_t)b * 32 + lane);
		const float amax = warp_max(fabsf(v));
		const float s1 = amax / 127.0f, s2 = s1 / 254.0f, s3 = s2 / 254.0f;
		int d1 = 0, d2 = 0, d3 = 0;
		if (s1 > 0.0f) {
			d1 = max(-127, min(127, __float2int_rn(v / s1)));
			const float q1 = __fmaf_rn(-(float)d1, s1, v);
			if (s2 > 0.0f) {
				d2 = max(-127, min(127, __float2int_rn(q1 / s2)));
				const float q2 = __fmaf_rn(-(float)d2, s2, q1);
				if (s3 > 0.0f)
					d3 = max(-127, min(127, __float2int_rn(q2 / s3)));
			}
		}
		int8_t *xb = reinterpret_cast<int8_t *>(xd + (size_t)b * kTcXd);
		xb[lane] = (int8_t)d1;
		xb[32 + lane] = (int8_t)d2;
		xb[64 + lane] = (int8_t)d3;
		const int t1 = __reduce_add_sync(0xffffffffu, d1);
		const int t2 = __reduce_add_sync(0xffffffffu, d2);
		const int t3 = __reduce_add_sync(0xffffffffu, d3);
		if (lane == 0) {
			pw[b * 4 + 0] = s1;
			pw[b * 4 + 1] = s2;
			pw[b * 4 + 2] = s3;
			pw[b * 4 + 3] = 0.0f;
			psum[b * 4 + 0] = t1;
			psum[b * 4 + 1] = t2;
			psum[b * 4 + 2] = t3;
			psum[b * 4 + 3] = 0;
		}
	}
	asm volatile("bar.sync 1, %0;" ::"n"(kTcMath * 32) : "memory");

	// MMA fragments: g = lane / 4 (rows g, g + 8; B column = digit plane g),
	// t = lane % 4 (codes 4t..4t+3 and 16+4t..; C columns 2t, 2t + 1)
	const int g = lane >> 2, t = lane & 3;
	// B: plane g < 3 of the block's digits, zeros for the unused columns
	const uint8_t *xbase = g < kTcPlanes ? xd + g * 32 + 4 * t : zero;
	const int xstride = g < kTcPlanes ? kTcXd : 0;
	// the plane scales and digit sums of this lane's C columns (2t, 2t + 1;
	// columns 3..7 are zero)
	const float *pwb = t < 2 ? pw + 2 * t : reinterpret_cast<const float *>(zero);
	const int32_t *psb = t < 2 ? psum + 2 * t : reinterpret_cast<const int32_t *>(zero);
	const int pstride = t < 2 ? 4 : 0;
	const int b_lo = warp * nb / kTcMath, b_hi = (warp + 1) * nb / kTcMath;
	bool failed = false;
	for (int i = 0; i < ntiles; i++) {
		const int slot = i % stages;
		if (!failed && !__all_sync(0xffffffffu, mbar_wait(&full[slot], (i / stages) & 1))) {
			failed = true;
			if (lane == 0 && err)
				atomicExch(err, 2);
		}
		float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // (g, 2t) (g, 2t+1) (g+8, 2t) (g+8, 2t+1)
		if (!failed) {
			const uint8_t *rg = ring + slot * tile_bytes + (int64_t)g * rs;
			const uint8_t *rg8 = rg + 8 * rs;
#pragma unroll 4
			for (int b = b_lo; b < b_hi; b++) {
				const uint8_t *pg = rg + b * BB, *pg8 = rg8 + b * BB;
				uint32_t a[4];
				if (QT == kQ8_0) {
					a[0] = lds_u32_a2(pg + 2 + 4 * t);
					a[1] = lds_u32_a2(pg8 + 2 + 4 * t);
					a[2] = lds_u32_a2(pg + 18 + 4 * t);
					a[3] = lds_u32_a2(pg8 + 18 + 4 * t);
				} else {
					// byte j: code j in the low nibble, code j + 16 in the high
					const uint32_t wg = lds_u32_a2(pg + 2 + 4 * t);
					const uint32_t wg8 = lds_u32_a2(pg8 + 2 + 4 * t);
					a[0] = wg & 0x0F0F0F0Fu;
					a[1] = wg8 & 0x0F0F0F0Fu;
					a[2] = (wg >> 4) & 0x0F0F0F0Fu;
					a[3] = (wg8 >> 4) & 0x0F0F0F0Fu;
				}
				const uint8_t *xb = xbase + (size_t)b * xstride;
				const uint32_t b0 = *reinterpret_cast<const uint32_t *>(xb);
				const uint32_t b1 = *reinterpret_cast<const uint32_t *>(xb + 16);
				int32_t dsum[4];
				imma_16832(dsum, a, b0, b1, QT == kQ4_0);
				if (QT == kQ4_0) {
					// codes were nib, values are nib - 8
					const int2 ps = *reinterpret_cast<const int2 *>(psb + (size_t)b * pstride);
					dsum[0] -= 8 * ps.x;
					dsum[1] -= 8 * ps.y;
					dsum[2] -= 8 * ps.x;
					dsum[3] -= 8 * ps.y;
				}
				const float2 sc = *reinterpret_cast<const float2 *>(pwb + (size_t)b * pstride);
				const float dg = half_bits_to_float(*reinterpret_cast<const uint16_t *>(pg));
				const float dg8 = half_bits_to_float(*reinterpret_cast<const uint16_t *>(pg8));
				acc[0] = __fmaf_rn((float)dsum[0], dg * sc.x, acc[0]);
				acc[1] = __fmaf_rn((float)dsum[1], dg * sc.y, acc[1]);
				acc[2] = __fmaf_rn((float)dsum[2], dg8 * sc.x, acc[2]);
				acc[3] = __fmaf_rn((float)dsum[3], dg8 * sc.y, acc[3]);
			}
		}
		__syncwarp();
		if (lane == 0)
			mbar_arrive(&empty[slot]);
		// this warp's share of rows g and g + 8: its columns (planes), then
		// the four lanes of the row
		float vg = acc[0] + acc[1], vg8 = acc[2] + acc[3];
		vg += __shfl_xor_sync(0xffffffffu, vg, 1);
		vg += __shfl_xor_sync(0xffffffffu, vg, 2);
		vg8 += __shfl_xor_sync(0xffffffffu, vg8, 1);
		vg8 += __shfl_xor_sync(0xffffffffu, vg8, 2);
		float *rd = red + (i & 1) * kTcMath * kTcRows + warp * kTcRows;
		if (t == 0) {
			rd[g] = vg;
			rd[g + 8] = vg8;
		}
		asm volatile("bar.sync 1, %0;" ::"n"(kTcMath * 32) : "memory");
		if (warp == 0 && lane < kTcRows) {
			const int r = r0 + i * kTcRows + lane;
			const float *rs = red + (i & 1) * kTcMath * kTcRows + lane;
			float v = 0.0f;
#pragma unroll
			for (int q = 0; q < kTcMath; q++)
				v += rs[q * kTcRows];
			if (r < r1)
				y[r] = v;
		}
	}
}

// ---------------------------------------------------------------- gemv1
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

// the ring's stages for a shape (0: the ring does not fit)
static int tc_stages(int qtype, int64_t cols)
{
	const int64_t rb = cols / QK * (qtype == kQ8_0 ? Q8_0_BYTES : Q4_0_BYTES);
	if (cols % 256 != 0 || rb % 16 != 0)
		return 0;
	for (int s = kTcMaxStages; s >= 2; s--)
		if (tc_smem(s, kTcRows * tc_row_stride(rb), (int)(cols / QK)) <= kTcSmemCap)
			return s;
	return 0;
}

bool gemv1_supported(int qtype, int64_t rows, int64_t cols, uintptr_t w, uintptr_t x, uintptr_t y)
{
	if (!((qtype == kQ8_0 || qtype == kQ4_0) && rows > 0 && rows <= INT32_MAX && cols > 0 &&
	      x % 16 == 0 && y % 4 == 0))
		return false;
	if (tc_stages(qtype, cols) && w % 16 == 0)
		return true;
	return cols % 64 == 0 && cols / QK * kXPad * 4 <= 200 * 1024 && w % 4 == 0;
}

template <int QT>
static cudaError_t launch_tc(const void *w, int64_t rows, int64_t cols, const float *x, float *y,
			     int32_t *err, int stages, cudaStream_t st)
{
	const int nb = (int)(cols / QK);
	const int64_t rb = (int64_t)nb * (QT == kQ8_0 ? Q8_0_BYTES : Q4_0_BYTES);
	const size_t smem = tc_smem(stages, kTcRows * tc_row_stride(rb), nb);
	cudaError_t e = ensure_smem(gemv_tc_kernel<QT>, smem);
	if (e != cudaSuccess)
		return e;
	int64_t grid = rows / kTcRows;
	if (grid > sm_count())
		grid = sm_count();
	if (grid < 1)
		grid = 1;
	gemv_tc_kernel<QT><<<(unsigned)grid, kTcThreads, smem, st>>>(
		static_cast<const uint8_t *>(w), (int)rows, nb, stages, x, y, err);
	return cudaGetLastError();
}

cudaError_t launch_gemv1(const void *w, int qtype, int64_t rows, int64_t cols, const float *x,
			 float *y, int32_t *err, cudaStream_t st)
{
	const int stages = tc_stages(qtype, cols);
	if (stages && (uintptr_t)w % 16 == 0)
		return qtype == kQ8_0 ? launch_tc<kQ8_0>(w, rows, cols, x, y, err, stages, st)
				      : launch_tc<kQ4_0>(w, rows, cols, x, y, err, stages, st);
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
