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
//   Each block's integer sums are exact; they become fp32 through the plane
//   scales and the block's fp16 weight scale (for Q4_0 a per-block constant
//   removes the nibble bias: minus 8 times the planes' digit sums).  The
//   three planes carry x to ~2^-17 of the block maximum, so the result is
//   within ~1e-6 relative of the reference's fp32 arithmetic (dot_f32_q4_0 /
//   dot_f32_q8_0, quant.c:103-155, which multiplies dequantized weights by
//   fp32 x).  Blocks are taken in pairs: every code word is one aligned
//   load or a funnel shift of two, and the odd block's planes sit in B
//   columns 4-6 (the even block's in 0-2), so its MMA accumulates onto the
//   even block's and one C tile, one conversion and one scale FMA per lane
//   and row serve both blocks (about 17 instructions per 16 rows x 32
//   codes); every shared-memory access is an explicit 32-bit-addressed
//   ld.shared.
// * 16 math warps split each tile's blocks (K) sixteen ways; partial row
//   sums meet in shared memory and are added in warp order.
// * Every CTA splits x into digits itself (16 KB of x, from L2) while its
//   first copies are in flight: each thread takes a quarter block (the 8
//   elements of one lane quad's B fragment), so the block maximum and the
//   digit sums are two shuffles and the 8 elements give the scheduler
//   independent work.
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
constexpr int kTcMath = 16;                     // math warps
constexpr int kTcThreads = (kTcMath + 1) * 32;  // + the copy warp
constexpr int kTcRows = 16;                     // rows per tile (the MMA's M)
constexpr int kTcPlanes = 3;                    // int8 digit planes of x (B columns 0..2)
constexpr int kTcMaxStages = 4;
constexpr size_t kTcSmemCap = 210 * 1024;
constexpr int kTcRedTiles = 8;                  // tiles per reduction of the partial row sums

// Shared memory after the stage ring, per block of x: the MMA B fragments
// [4 t][8 g][8 bytes] (lane (g, t) reads its b0, b1 as one 8-byte word;
// planes in columns 0-2 for an even block, 4-6 for an odd one, the other
// columns zero) = 256 bytes, and the plane weights [4 t][4] f32 = (weight,
// 0, nibble correction, 0) = 64 bytes; then the partial sums
// [kTcRedTiles][kTcMath][16] f32 and the mbarriers.  Lane quad t's C columns (2t,
// 2t + 1) combine in integers as 254 c_2t + c_2t+1 (|.| < 2^27, exact) and
// take one weight: s2 for planes 0-1, s3 / 254 for plane 2.
constexpr int kTcB = 256, kTcW = 64, kTcPerBlock = kTcB + kTcW;

// bytes between rows in a stage: rows of 4096 (Q4_0) or 2048 (Q8_0) columns
// are multiples of 128 bytes, so unpadded, the eight rows one fragment load
// touches would all fall in the same shared-memory bank
__host__ __device__ inline int64_t tc_row_stride(int64_t rb) { return rb + 16; }
inline size_t tc_smem(int stages, int64_t tile_bytes, int nb)
{
	return (size_t)stages * tile_bytes + (size_t)nb * kTcPerBlock +
	       kTcRedTiles * kTcMath * kTcRows * 4 + 2 * kTcMaxStages * 8;
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

// the same product added onto d
__device__ __forceinline__ void imma_16832_acc(int32_t (&d)[4], const uint32_t (&a)[4],
					       uint32_t b0, uint32_t b1, bool a_unsigned)
{
	if (a_unsigned)
		asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
			     "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
			     : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
			     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
	else
		asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
			     "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
			     : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
			     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// shared-memory loads by 32-bit shared address (every access to the stage
// ring and the x fragments is an explicit ld.shared)
__device__ __forceinline__ uint2 lds64(uint32_t a)
{
	uint2 v;
	asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
	return v;
}
__device__ __forceinline__ float4 lds128f(uint32_t a)
{
	float4 v;
	asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
		     : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
		     : "r"(a));
	return v;
}

constexpr int kTcMaxXb = 14;  // blocks of x per math warp (cols / 32 / kTcMath at most)


// shared-memory loads at a register address plus a compile-time offset
template <int OFF>
__device__ __forceinline__ uint32_t lds32o(uint32_t a)
{
	uint32_t v;
	asm volatile("ld.shared.b32 %0, [%1+%2];" : "=r"(v) : "r"(a), "n"(OFF));
	return v;
}
template <int OFF>
__device__ __forceinline__ float lds_half_o(uint32_t a)
{
	unsigned short h;
	asm volatile("ld.shared.u16 %0, [%1+%2];" : "=h"(h) : "r"(a), "n"(OFF));
	return __half2float(__ushort_as_half(h));
}

// A fragments of two adjacent blocks (the pair starting OFF bytes after a
// 4-byte aligned row position; `a` = that position + 4t for lane quad t):
// codes 4t..4t+3 (lo) and 16+4t..16+4t+3 (hi) of each block.  Q4_0 (2 x 18
// bytes): byte j of a block holds code j (low nibble) and code j + 16 (high
// nibble); the even block's code bytes start 2 bytes past a word, the odd
// block's on one.  Q8_0 (2 x 34 bytes): int8 codes at the same offsets.
template <int QT, int OFF>
__device__ __forceinline__ void pair_codes(uint32_t a, uint32_t (&ev)[2], uint32_t (&od)[2])
{
	if (QT == kQ4_0) {
		const uint32_t e = __funnelshift_r(lds32o<OFF>(a), lds32o<OFF + 4>(a), 16);
		const uint32_t o = lds32o<OFF + 20>(a);
		ev[0] = e & 0x0F0F0F0Fu;
		ev[1] = (e >> 4) & 0x0F0F0F0Fu;
		od[0] = o & 0x0F0F0F0Fu;
		od[1] = (o >> 4) & 0x0F0F0F0Fu;
	} else {
		ev[0] = __funnelshift_r(lds32o<OFF>(a), lds32o<OFF + 4>(a), 16);
		ev[1] = __funnelshift_r(lds32o<OFF + 16>(a), lds32o<OFF + 20>(a), 16);
		od[0] = lds32o<OFF + 36>(a);
		od[1] = lds32o<OFF + 52>(a);
	}
}

// Expert segments (SegMap with wtab set): the grid is split into units
// (column chunk, activation row), the CTAs of a unit into row ranges of its
// segments placed end to end.  Row r of a unit: segment r / rows, row
// r % rows of that matrix, its chunk `c` of nb blocks.
struct SegPos {
	int c, xi;     // column chunk, activation row (down: the slot)
	int nseg;      // segments of the unit (gate/up: 2K, down: 1)
};

__device__ __forceinline__ const uint8_t *seg_row(const SegMap &sm, const SegPos &p, int rows,
						  int r, int64_t rb)
{
	const int sl = r / rows, rr = r - sl * rows;
	const int slot = sm.down ? p.xi : (sl < sm.K ? sl : sl - sm.K);
	const int kind = sm.down ? 2 : (sl < sm.K ? 0 : 1);
	const uint8_t *base = static_cast<const uint8_t *>(sm.wtab[kind * sm.NE + sm.ids[slot]]);
	return base + (int64_t)rr * sm.rb_full + (int64_t)p.c * rb;
}

// NBW: blocks of a row per math warp (cols / 32 / kTcMath, even)
template <int QT, int NBW>
__global__ void __launch_bounds__(kTcThreads, 1)
gemv_tc_kernel(const uint8_t *__restrict__ w, int rows, int nb, int stages,
	       const float *__restrict__ x, float *__restrict__ y, int32_t *err, NormIn nin,
	       SegMap sm)
{
	constexpr int BB = QT == kQ8_0 ? Q8_0_BYTES : Q4_0_BYTES;
	extern __shared__ __align__(128) uint8_t smem[];
	const int64_t rb = (int64_t)nb * BB;          // row bytes (a multiple of 16)
	const int64_t rs = tc_row_stride(rb);         // row stride in a stage
	const int64_t tile_bytes = kTcRows * rs;
	uint8_t *ring = smem;
	uint8_t *xfrag = smem + stages * tile_bytes;                 // [nb][kTcB]
	uint8_t *xw = xfrag + (size_t)nb * kTcB;                      // [nb][kTcW]
	float *red = reinterpret_cast<float *>(xw + (size_t)nb * kTcW);  // [kTcRedTiles][kTcMath][16]
	uint64_t *full = reinterpret_cast<uint64_t *>(red + kTcRedTiles * kTcMath * kTcRows);
	uint64_t *empty = full + kTcMaxStages;

	const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
	int r0 = (int)((int64_t)blockIdx.x * rows / gridDim.x);
	int r1 = (int)((int64_t)(blockIdx.x + 1) * rows / gridDim.x);
	SegPos sp{0, 0, 1};
	if (sm.wtab) {
		// the slots' experts (and the weights they select) come from the
		// kernel before: launched as its dependent, wait for it first
		griddep_wait();
		// this CTA's unit and its row range in the unit's segments
		const int nx = sm.down ? sm.K : 1, U = sm.nchunks * nx, G = (int)gridDim.x;
		const int u = (int)((int64_t)blockIdx.x * U / G);
		const int b0u = (int)(((int64_t)u * G + U - 1) / U);
		const int b1u = (int)(((int64_t)(u + 1) * G + U - 1) / U);
		sp.c = u % sm.nchunks;
		sp.xi = u / sm.nchunks;
		sp.nseg = sm.down ? 1 : 2 * sm.K;
		const int64_t R = (int64_t)sp.nseg * rows;
		const int i = (int)blockIdx.x - b0u, n = b1u - b0u;
		r0 = (int)(i * R / n);
		r1 = (int)((i + 1) * R / n);
		if (rows % 2 == 0) {
			// even bounds: a row pair never spans two matrices
			r0 &= ~1;
			r1 = i + 1 == n ? (int)R : (r1 & ~1);
		}
		// a slot's expert out of range: flag it, compute nothing
		bool bad = false;
		for (int k = 0; k < sm.K; k++)
			bad |= (unsigned)sm.ids[k] >= (unsigned)sm.NE;
		if (bad) {
			if (tid == 0 && err)
				atomicExch(err, 1);
			return;
		}
	}
	const int ntiles = (r1 - r0 + kTcRows - 1) / kTcRows;
	// rows adjacent in memory (not a column chunk of a wider matrix): one
	// bulk copy per row pair (2 rb bytes, pair j at j (2 rb + 16) in the
	// stage), MMA rows g and g + 8 being the tile's rows 2g and 2g + 1; the
	// copy engine takes a request every ~0.1 us per SM, which bounded the
	// stream at one request per row.  Else one copy per row at j rs.
	const bool pairs = !sm.wtab || sm.nchunks == 1;
	const int64_t ps = 2 * rb + 16;  // pair stride
	if (tid == 0) {
		for (int i = 0; i < stages; i++) {
			mbar_init(&full[i], 1);
			mbar_init(&empty[i], kTcMath);
		}
		fence_mbar_init();
	}
	__syncthreads();
	// launched as a dependent (model decode step): the next kernel may start
	// its own prologue now; this one streams its (constant) weights at once
	// and waits for the earlier kernel only before reading x
	griddep_launch_dependents();

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
			if (pairs) {
				if (2 * lane < n) {
					const int nr = min(2, n - 2 * lane);
					const uint8_t *src = sm.wtab ? seg_row(sm, sp, rows, r + 2 * lane, rb)
								     : w + (int64_t)(r + 2 * lane) * rb;
					fence_proxy_async();
					bulk_g2s(ring + slot * tile_bytes + lane * ps, src, (uint32_t)(nr * rb),
						 &full[slot]);
				}
			} else if (lane < n) {
				const uint8_t *src = sm.wtab ? seg_row(sm, sp, rows, r + lane, rb)
							     : w + (int64_t)(r + lane) * rb;
				fence_proxy_async();
				bulk_g2s(ring + slot * tile_bytes + lane * rs, src, (uint32_t)rb, &full[slot]);
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

	// ---- math warps.  x as three int8 digit planes per block.  Thread q of
	// the math warps takes quarter q % 4 of block q / 4 (and q + 512, ...):
	// elements 4 (q % 4) + {0..3} and 16 + 4 (q % 4) + {0..3}, which are
	// exactly the 8 bytes of each plane's B fragment for lane quad q % 4,
	// so every plane leaves as one 8-byte store.  The block maximum and the
	// digit sums are two shuffles among the block's 4 (adjacent) threads, and
	// a thread's 8 elements are independent, so the prologue is short and
	// issues densely (a whole warp per block, with a warp-wide reduction
	// between dependent steps, took ~0.4 us per block).
	{
		constexpr int QPT = (NBW + 7) / 8;  // quarters per thread: nb * 4 = 64 NBW over 512
		const int nq = nb * 4;              // a multiple of 64: whole warps active or not
		float va[QPT][8];
		griddep_wait();
		// this thread's elements of quarter it: e0 + {0..3}, e0 + 16 + {0..3}
		auto ld8 = [&](const float *p, int e0, float (&o)[8], bool coherent) {
			if (((uintptr_t)p & 15) == 0) {
				const float4 u0 = coherent ? __ldcg(reinterpret_cast<const float4 *>(p + e0))
							   : __ldg(reinterpret_cast<const float4 *>(p + e0));
				const float4 u1 = coherent ? __ldcg(reinterpret_cast<const float4 *>(p + e0 + 16))
							   : __ldg(reinterpret_cast<const float4 *>(p + e0 + 16));
				o[0] = u0.x; o[1] = u0.y; o[2] = u0.z; o[3] = u0.w;
				o[4] = u1.x; o[5] = u1.y; o[6] = u1.z; o[7] = u1.w;
			} else {
#pragma unroll
				for (int e = 0; e < 8; e++)
					o[e] = coherent ? __ldcg(p + e0 + (e & 3) + (e >> 2) * 16)
							: __ldg(p + e0 + (e & 3) + (e >> 2) * 16);
			}
		};
		if (nin.hidden) {
			// x = rms_norm(hidden + delta) * weight (tensor_add, then
			// rms_norm, nn.c:7-48); CTA 0 stores hidden + delta.  Every
			// load comes before the first store (hidden_out might alias
			// them as far as the compiler knows).
			float dl[QPT][8], wn[QPT][8];
#pragma unroll
			for (int it = 0; it < QPT; it++) {
				const int q = tid + it * kTcMath * 32;
				if (q < nq) {
					const int e0 = (q >> 2) * 32 + 4 * (q & 3);
					ld8(nin.hidden, e0, va[it], true);
					if (nin.delta)
						ld8(nin.delta, e0, dl[it], true);
					ld8(nin.weight, e0, wn[it], false);
				}
			}
			float ss = 0.0f;
#pragma unroll
			for (int it = 0; it < QPT; it++) {
				const int q = tid + it * kTcMath * 32;
				if (q < nq) {
					const int e0 = (q >> 2) * 32 + 4 * (q & 3);
#pragma unroll
					for (int e = 0; e < 8; e++) {
						if (nin.delta)
							va[it][e] = __fadd_rn(va[it][e], dl[it][e]);
						if (blockIdx.x == 0)
							nin.hidden_out[e0 + (e & 3) + (e >> 2) * 16] = va[it][e];
						ss = fmaf(va[it][e], va[it][e], ss);
					}
				}
			}
			ss = warp_sum(ss);
			if (lane == 0)
				red[warp] = ss;
			asm volatile("bar.sync 1, %0;" ::"n"(kTcMath * 32) : "memory");
			float tot = 0.0f;
#pragma unroll
			for (int q = 0; q < kTcMath; q++)
				tot += red[q];
			const float rms = sqrtf(tot / (float)(nb * 32) + nin.eps);
#pragma unroll
			for (int it = 0; it < QPT; it++)
#pragma unroll
				for (int e = 0; e < 8; e++)
					va[it][e] = (va[it][e] / rms) * wn[it][e];
		} else if (sm.wtab && sm.down) {
			// h of this unit's slot: swiglu(gate row, up row) (nn.c:475-478)
			const int64_t cols = (int64_t)sm.nchunks * nb * 32;
			const float *gp = sm.gu + (int64_t)sp.xi * cols + (int64_t)sp.c * nb * 32;
			const float *up = gp + (int64_t)sm.K * cols;
#pragma unroll
			for (int it = 0; it < QPT; it++) {
				const int q = tid + it * kTcMath * 32;
				if (q < nq) {
					const int e0 = (q >> 2) * 32 + 4 * (q & 3);
					float gv[8], uv[8];
					ld8(gp, e0, gv, true);
					ld8(up, e0, uv, true);
#pragma unroll
					for (int e = 0; e < 8; e++)
						va[it][e] = swiglu(gv[e], uv[e]);
				}
			}
		} else {
			const float *xc = x + (int64_t)sp.c * nb * 32;
#pragma unroll
			for (int it = 0; it < QPT; it++) {
				const int q = tid + it * kTcMath * 32;
				if (q < nq)
					ld8(xc, (q >> 2) * 32 + 4 * (q & 3), va[it], false);
			}
		}
#pragma unroll
		for (int it = 0; it < QPT; it++) {
			const int q = tid + it * kTcMath * 32;
			if (q >= nq)
				continue;   // whole warps (nq is a multiple of 64)
			const int b = q >> 2, tq = q & 3;
			float am = 0.0f;
#pragma unroll
			for (int e = 0; e < 8; e++)
				am = fmaxf(am, fabsf(va[it][e]));
			am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
			const float amax = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
			float s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
			int d1[8], d2[8], d3[8];
#pragma unroll
			for (int e = 0; e < 8; e++)
				d1[e] = d2[e] = d3[e] = 0;
			if (amax > 0.0f) {
				// the digits only need s * d to track x: every residual is
				// taken exactly (fma) against the same s, so an approximate
				// reciprocal serves instead of a division (a digit that
				// rounds the other way leaves a residual the next plane
				// takes; the clamps keep every digit in range)
				s1 = amax * (1.0f / 127.0f);
				s2 = s1 * (1.0f / 254.0f);
				s3 = s2 * (1.0f / 254.0f);
				const float i1 = __fdividef(1.0f, s1), i2 = i1 * 254.0f, i3 = i2 * 254.0f;
#pragma unroll
				for (int e = 0; e < 8; e++) {
					const float v = va[it][e];
					d1[e] = max(-127, min(127, __float2int_rn(v * i1)));
					const float q1 = __fmaf_rn(-(float)d1[e], s1, v);
					d2[e] = max(-127, min(127, __float2int_rn(q1 * i2)));
					const float q2 = __fmaf_rn(-(float)d2[e], s2, q1);
					d3[e] = (s3 > 0.0f) ? max(-127, min(127, __float2int_rn(q2 * i3))) : 0;
				}
			}
			// each plane's 8 digits as the two words b0 (elements 4tq..) and
			// b1 (16 + 4tq..) of its B fragment
			auto pack = [](const int (&d)[8], int o) {
				return __byte_perm(__byte_perm(d[o], d[o + 1], 0x0040),
						   __byte_perm(d[o + 2], d[o + 3], 0x0040), 0x5410);
			};
			const uint2 w1 = make_uint2(pack(d1, 0), pack(d1, 4));
			const uint2 w2 = make_uint2(pack(d2, 0), pack(d2, 4));
			const uint2 w3 = make_uint2(pack(d3, 0), pack(d3, 4));
			// B fragment bytes: [t][column g][b0 | b1].  An even block's
			// planes are columns 0-2, an odd block's columns 4-6 (the other
			// columns zero), so the MMA of an odd block can accumulate onto
			// its even neighbour's and both leave one C tile.
			const int cb = (b & 1) * 4;
			uint2 *fb = reinterpret_cast<uint2 *>(xfrag + (size_t)b * kTcB + tq * 64);
#pragma unroll
			for (int c = 0; c < 8; c++) {
				const int pl = (c - cb) & 7;   // plane of column c (none past the planes)
				fb[c] = pl >= kTcPlanes ? make_uint2(0, 0) : pl == 0 ? w1 : pl == 1 ? w2 : w3;
			}
			// digit sums of the planes over the block (signed bytes)
			int S1 = __dp4a((int)w1.x, 0x01010101, __dp4a((int)w1.y, 0x01010101, 0));
			int S2 = __dp4a((int)w2.x, 0x01010101, __dp4a((int)w2.y, 0x01010101, 0));
			int S3 = __dp4a((int)w3.x, 0x01010101, __dp4a((int)w3.y, 0x01010101, 0));
			S1 += __shfl_xor_sync(0xffffffffu, S1, 1);
			S2 += __shfl_xor_sync(0xffffffffu, S2, 1);
			S3 += __shfl_xor_sync(0xffffffffu, S3, 1);
			S1 += __shfl_xor_sync(0xffffffffu, S1, 2);
			S2 += __shfl_xor_sync(0xffffffffu, S2, 2);
			S3 += __shfl_xor_sync(0xffffffffu, S3, 2);
			// entry tq = (w_2t, 0, nibble correction, 0): the weight of lane
			// quad t's combined C columns and, once per block, minus 8 x the
			// planes' digit sums (Q4_0 codes are nib, their values nib - 8).
			// Quads 0-1 read an even block's entries, quads 2-3 an odd
			// block's: the first of its quads holds planes 0 and 1, combined
			// exactly in integers as 254 D0 + D1 with the weight s2 (= s1 /
			// 254 to fp32 rounding); the second holds plane 2 (and an empty
			// column) as 254 D2 with the weight s3 / 254.
			const float corr =
				QT == kQ4_0 ? -8.0f * ((float)S1 * s1 + (float)S2 * s2 + (float)S3 * s3) : 0.0f;
			const int qq = tq - (b & 1) * 2;   // 0, 1: this block's quads
			reinterpret_cast<float4 *>(xw + (size_t)b * kTcW)[tq] = make_float4(
				qq == 0 ? s2 : (qq == 1 ? s3 / 254.0f : 0.0f), 0.0f, qq == 0 ? corr : 0.0f, 0.0f);
		}
	}
	asm volatile("bar.sync 1, %0;" ::"n"(kTcMath * 32) : "memory");

	// MMA fragments: g = lane / 4 (rows g, g + 8; B column = digit plane g),
	// t = lane % 4 (codes 4t..4t+3 and 16+4t..; C columns 2t, 2t + 1).  This
	// warp's blocks [NBW*warp, +NBW): their B fragments and plane weights
	// stay in registers for every tile.
	const int g = lane >> 2, t = lane & 3;
	const int b0 = warp * NBW;
	uint2 bfr[NBW];
	// quads 0-1 weigh the even block of each pair, quads 2-3 the odd one
	float wx[NBW / 2], wz[NBW / 2];
#pragma unroll
	for (int j = 0; j < NBW; j++)
		bfr[j] = lds64(smem_addr(xfrag) + (uint32_t)((b0 + j) * kTcB + t * 64 + g * 8));
#pragma unroll
	for (int jp = 0; jp < NBW / 2; jp++) {
		const float4 wv =
			lds128f(smem_addr(xw) + (uint32_t)((b0 + 2 * jp + (t >> 1)) * kTcW + t * 16));
		wx[jp] = wv.x;
		wz[jp] = wv.z;
	}
	const uint32_t s_row =
		smem_addr(ring) + (uint32_t)((pairs ? g * ps : g * rs) + b0 * BB);
	const uint32_t d8 = (uint32_t)(pairs ? rb : 8 * rs);  // MMA row g + 8 from row g
	const uint32_t so = (uint32_t)((t >> 1) * BB);        // this quad's block scale
	bool failed = false;
	for (int i = 0; i < ntiles; i++) {
		const int slot = i % stages;
		if (!failed && !__all_sync(0xffffffffu, mbar_wait(&full[slot], (i / stages) & 1))) {
			failed = true;
			if (lane == 0 && err)
				atomicExch(err, 2);
		}
		float acc_g = 0.0f, acc_g8 = 0.0f;
		if (!failed) {
			// rows g and g + 8 of this stage at this warp's first block
			const uint32_t rg = s_row + (uint32_t)(slot * tile_bytes);
			const uint32_t rg8 = rg + d8;
			static_for<NBW / 2>([&](auto J) {
				constexpr int jp = decltype(J)::value;
				constexpr int OFF = 2 * jp * BB;
				uint32_t eg[2], og[2], eg8[2], og8[2];
				pair_codes<QT, OFF>(rg + 4 * t, eg, og);
				pair_codes<QT, OFF>(rg8 + 4 * t, eg8, og8);
				// the scale of this quad's block (even: quads 0-1, odd: 2-3)
				const float dg = lds_half_o<OFF>(rg + so), d8 = lds_half_o<OFF>(rg8 + so);
				const uint32_t ae[4] = {eg[0], eg8[0], eg[1], eg8[1]};
				const uint32_t ao[4] = {og[0], og8[0], og[1], og8[1]};
				// the odd block's sums (columns 4-7) accumulate onto the even
				// block's (columns 0-3): one C tile holds both blocks
				int32_t c[4];
				imma_16832(c, ae, bfr[2 * jp].x, bfr[2 * jp].y, QT == kQ4_0);
				imma_16832_acc(c, ao, bfr[2 * jp + 1].x, bfr[2 * jp + 1].y, QT == kQ4_0);
				acc_g = __fmaf_rn(dg, __fmaf_rn((float)(c[0] * 254 + c[1]), wx[jp], wz[jp]),
						  acc_g);
				acc_g8 = __fmaf_rn(d8, __fmaf_rn((float)(c[2] * 254 + c[3]), wx[jp], wz[jp]),
						   acc_g8);
			});
		}
		__syncwarp();
		if (lane == 0)
			mbar_arrive(&empty[slot]);
		// this warp's share of rows g and g + 8: the four lanes of the row
		acc_g += __shfl_xor_sync(0xffffffffu, acc_g, 1);
		acc_g += __shfl_xor_sync(0xffffffffu, acc_g, 2);
		acc_g8 += __shfl_xor_sync(0xffffffffu, acc_g8, 1);
		acc_g8 += __shfl_xor_sync(0xffffffffu, acc_g8, 2);
		// partial sums of up to kTcRedTiles tiles wait in shared memory; the
		// math warps meet once per chunk of tiles (not once per tile) and
		// then add the chunk's rows in warp order, one row per thread
		const int ct = i % kTcRedTiles;
		float *rd = red + (ct * kTcMath + warp) * kTcRows;
		if (t == 0) {
			rd[g] = acc_g;
			rd[g + 8] = acc_g8;
		}
		if (ct == kTcRedTiles - 1 || i == ntiles - 1) {
			asm volatile("bar.sync 1, %0;" ::"n"(kTcMath * 32) : "memory");
			const int n = (ct + 1) * kTcRows;   // rows of this chunk
			if (tid < n) {
				const int m = tid % kTcRows;    // MMA row -> its tile row
				const int tr = pairs ? (m < 8 ? 2 * m : 2 * m - 15) : m;
				const int r = r0 + (i - ct + tid / kTcRows) * kTcRows + tr;
				const float *rsum = red + (tid / kTcRows) * kTcMath * kTcRows + m;
				float v = 0.0f;
#pragma unroll
				for (int q = 0; q < kTcMath; q++)
					v += rsum[q * kTcRows];
				if (r < r1) {
					if (sm.wtab) {
						const int sl = r / rows, rr = r - sl * rows;
						const int s_ = sm.down ? sp.xi : sl;
						const int nsg = sm.down ? sm.K : 2 * sm.K;
						sm.part[((int64_t)sp.c * nsg + s_) * rows + rr] = v;
					} else {
						y[r] = v;
					}
				}
			}
			// the next chunk overwrites these partial sums
			asm volatile("bar.sync 1, %0;" ::"n"(kTcMath * 32) : "memory");
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
	// an even number of blocks per math warp, at most kTcMaxXb
	if (cols % (32 * 2 * kTcMath) != 0 || cols / QK > kTcMath * kTcMaxXb || rb % 16 != 0)
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

template <int QT, int NBW>
static cudaError_t launch_tc_t(const void *w, int64_t rows, int nb, const float *x, float *y,
			       int32_t *err, int stages, size_t smem, const NormIn &nin, bool pdl,
			       cudaStream_t st)
{
	auto fn = gemv_tc_kernel<QT, NBW>;
	cudaError_t e = ensure_smem(fn, smem);
	if (e != cudaSuccess)
		return e;
	int64_t grid = rows / kTcRows;
	if (grid > sm_count())
		grid = sm_count();
	if (grid < 1)
		grid = 1;
	cudaLaunchConfig_t cfg{};
	cfg.gridDim = dim3((unsigned)grid);
	cfg.blockDim = dim3(kTcThreads);
	cfg.dynamicSmemBytes = smem;
	cfg.stream = st;
	cudaLaunchAttribute at[1];
	at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	at[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = at;
	cfg.numAttrs = pdl ? 1 : 0;
	return cudaLaunchKernelEx(&cfg, fn, static_cast<const uint8_t *>(w), (int)rows, nb, stages,
				  x, y, err, nin, SegMap{});
}

template <int QT>
static cudaError_t launch_tc(const void *w, int64_t rows, int64_t cols, const float *x, float *y,
			     int32_t *err, int stages, const NormIn &nin, bool pdl, cudaStream_t st)
{
	const int nb = (int)(cols / QK);
	const int64_t rb = (int64_t)nb * (QT == kQ8_0 ? Q8_0_BYTES : Q4_0_BYTES);
	const size_t smem = tc_smem(stages, kTcRows * tc_row_stride(rb), nb);
	switch (nb / kTcMath) {
	case 2:
		return launch_tc_t<QT, 2>(w, rows, nb, x, y, err, stages, smem, nin, pdl, st);
	case 4:
		return launch_tc_t<QT, 4>(w, rows, nb, x, y, err, stages, smem, nin, pdl, st);
	case 6:
		return launch_tc_t<QT, 6>(w, rows, nb, x, y, err, stages, smem, nin, pdl, st);
	case 8:
		return launch_tc_t<QT, 8>(w, rows, nb, x, y, err, stages, smem, nin, pdl, st);
	case 10:
		return launch_tc_t<QT, 10>(w, rows, nb, x, y, err, stages, smem, nin, pdl, st);
	case 12:
		return launch_tc_t<QT, 12>(w, rows, nb, x, y, err, stages, smem, nin, pdl, st);
	case 14:
		return launch_tc_t<QT, 14>(w, rows, nb, x, y, err, stages, smem, nin, pdl, st);
	default:
		return cudaErrorInvalidValue;
	}
}

// ---------------------------------------------------------------- one token's experts
template <int QT, int NBW>
static cudaError_t launch_seg_t(int rows, int nb, const float *x, int32_t *err, int stages,
				size_t smem, const SegMap &sm, cudaStream_t st)
{
	auto fn = gemv_tc_kernel<QT, NBW>;
	cudaError_t e = ensure_smem(fn, smem);
	if (e != cudaSuccess)
		return e;
	// a programmatic dependent of the kernel before (it waits for it before
	// reading the experts, x or h)
	cudaLaunchConfig_t cfg{};
	cfg.gridDim = dim3((unsigned)sm_count());
	cfg.blockDim = dim3(kTcThreads);
	cfg.dynamicSmemBytes = smem;
	cfg.stream = st;
	cudaLaunchAttribute at[1];
	at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	at[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = at;
	cfg.numAttrs = pdl_enabled() ? 1 : 0;
	return cudaLaunchKernelEx(&cfg, fn, static_cast<const uint8_t *>(nullptr), rows, nb, stages, x,
				  static_cast<float *>(nullptr), err, NormIn{}, sm);
}

template <int QT>
static cudaError_t launch_seg(int rows, int64_t cols, const float *x, int32_t *err,
			      const SegMap &sm, cudaStream_t st)
{
	const int stages = tc_stages(QT, cols);
	if (!stages)
		return cudaErrorNotSupported;
	const int nb = (int)(cols / QK);
	const int64_t rb = (int64_t)nb * (QT == kQ8_0 ? Q8_0_BYTES : Q4_0_BYTES);
	const size_t smem = tc_smem(stages, kTcRows * tc_row_stride(rb), nb);
	switch (nb / kTcMath) {
	case 2:
		return launch_seg_t<QT, 2>(rows, nb, x, err, stages, smem, sm, st);
	case 4:
		return launch_seg_t<QT, 4>(rows, nb, x, err, stages, smem, sm, st);
	case 6:
		return launch_seg_t<QT, 6>(rows, nb, x, err, stages, smem, sm, st);
	case 8:
		return launch_seg_t<QT, 8>(rows, nb, x, err, stages, smem, sm, st);
	case 10:
		return launch_seg_t<QT, 10>(rows, nb, x, err, stages, smem, sm, st);
	case 12:
		return launch_seg_t<QT, 12>(rows, nb, x, err, stages, smem, sm, st);
	case 14:
		return launch_seg_t<QT, 14>(rows, nb, x, err, stages, smem, sm, st);
	default:
		return cudaErrorInvalidValue;
	}
}

// out = sum over slots k (in slot order) of y_k / (1 / w_k), y_k the sum of
// its column chunks' partial rows in chunk order (the combine of
// olmoe.c:387-405 with the reciprocal division of the other paths)
__global__ void t1_combine_kernel(const float *__restrict__ part, const float *__restrict__ w,
				  int nchunks, int K, int D, float *__restrict__ out)
{
	griddep_launch_dependents();
	griddep_wait();
	const int j = blockIdx.x * blockDim.x + threadIdx.x;
	if (j >= D)
		return;
	float acc = 0.0f;
	for (int k = 0; k < K; k++) {
		float y = part[(int64_t)k * D + j];
		for (int c = 1; c < nchunks; c++)
			y = __fadd_rn(y, part[((int64_t)c * K + k) * D + j]);
		acc = __fadd_rn(__fdiv_rn(y, __fdiv_rn(1.0f, w[k])), acc);
	}
	out[j] = acc;
}

int expert_t1_chunks(int qtype, int64_t D, int64_t F, int K)
{
	if ((qtype != kQ8_0 && qtype != kQ4_0) || K < 1 || K > 32 || !tc_stages(qtype, D) ||
	    F > INT32_MAX / 2 || D > INT32_MAX / 2)
		return 0;
	// the largest chunk of whole 1024-column groups that the ring fits
	for (int64_t n = 1; n <= 64; n++) {
		if (F % n != 0 || (F / n) % 1024 != 0)
			continue;
		if (tc_stages(qtype, F / n))
			return n * K <= sm_count() ? (int)n : 0;
	}
	return 0;
}

cudaError_t launch_expert_t1(int stage, const void *const *wtab, const int32_t *ids,
			     const float *w, int qtype, int64_t D, int64_t F, int NE, int K,
			     const float *x, float *gu, float *part, float *out, int32_t *err,
			     cudaStream_t st)
{
	const int nch = expert_t1_chunks(qtype, D, F, K);
	if (!nch)
		return cudaErrorNotSupported;
	const int BB = qtype == kQ8_0 ? Q8_0_BYTES : Q4_0_BYTES;
	SegMap a;
	a.wtab = wtab;
	a.ids = ids;
	a.NE = NE;
	a.K = K;
	if (stage == 0) {
		a.down = 0;
		a.nchunks = 1;
		a.rb_full = D / QK * BB;
		a.part = gu;
		return qtype == kQ8_0 ? launch_seg<kQ8_0>((int)F, D, x, err, a, st)
				      : launch_seg<kQ4_0>((int)F, D, x, err, a, st);
	}
	if (stage == 1) {
		a.down = 1;
		a.nchunks = nch;
		a.rb_full = F / QK * BB;
		a.gu = gu;
		a.part = part;
		return qtype == kQ8_0 ? launch_seg<kQ8_0>((int)D, F / nch, nullptr, err, a, st)
				      : launch_seg<kQ4_0>((int)D, F / nch, nullptr, err, a, st);
	}
	cudaLaunchConfig_t cfg{};
	cfg.gridDim = dim3((unsigned)((D + 255) / 256));
	cfg.blockDim = dim3(256);
	cfg.stream = st;
	cudaLaunchAttribute at[1];
	at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	at[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = at;
	cfg.numAttrs = pdl_enabled() ? 1 : 0;
	return cudaLaunchKernelEx(&cfg, t1_combine_kernel, static_cast<const float *>(part), w, nch, K,
				  (int)D, out);
}

bool gemv_norm_supported(int qtype, int64_t cols, uintptr_t w)
{
	return (qtype == kQ8_0 || qtype == kQ4_0) && tc_stages(qtype, cols) && w % 16 == 0;
}

cudaError_t launch_gemv_norm(const void *w, int qtype, int64_t rows, int64_t cols,
			     const NormIn &nin, float *y, int32_t *err, bool pdl, cudaStream_t st)
{
	const int stages = tc_stages(qtype, cols);
	if (!stages || (uintptr_t)w % 16 || !nin.hidden || !nin.weight || !nin.hidden_out)
		return cudaErrorNotSupported;
	return qtype == kQ8_0 ? launch_tc<kQ8_0>(w, rows, cols, nullptr, y, err, stages, nin, pdl, st)
			      : launch_tc<kQ4_0>(w, rows, cols, nullptr, y, err, stages, nin, pdl, st);
}

cudaError_t launch_gemv1(const void *w, int qtype, int64_t rows, int64_t cols, const float *x,
			 float *y, int32_t *err, cudaStream_t st, bool pdl)
{
	const int stages = tc_stages(qtype, cols);
	if (stages && (uintptr_t)w % 16 == 0)
		return qtype == kQ8_0 ? launch_tc<kQ8_0>(w, rows, cols, x, y, err, stages, NormIn{}, pdl, st)
				      : launch_tc<kQ4_0>(w, rows, cols, x, y, err, stages, NormIn{}, pdl, st);
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
