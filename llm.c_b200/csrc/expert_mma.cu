// expert_mma.cu — decode-time grouped expert GEMV/GEMM on the tensor cores.
//
// Work: for every expert e with n_e routed (token, slot) pairs, stream the
// expert's Q8_0/Q4_0 weight rows from HBM once and multiply them with the
// n_e activation rows (fused SwiGLU for gate/up, plain for down).  This is
// the memory-bound regime (n_e is ~1-32 at decode), so the kernel is built
// around moving bytes:
//
//  * Warps are persistent and independent: each takes (expert, row group)
//    items from a global counter and runs its own copy pipeline, in which
//    lane l copies row l's next 8-block chunk (272 B of Q8_0, 144 B of
//    Q4_0; GGUF rows are a multiple of 16 B when cols % 256 == 0) into
//    shared memory with cp.async.bulk, completing on a per-stage mbarrier.
//    No block-wide barrier is ever taken, so warps drift freely and keep
//    HBM busy; 16 warps per SM hide the dependent-MMA latency.
//  * The int8 (or 4-bit) codes are turned into exact fp16 integers with a
//    byte permute (q ^ 0x80 placed under the fp16 exponent of 1024, minus
//    1152), so a weight byte costs about two instructions.
//  * mma.sync m16n8k16 multiplies them with the activations split into two
//    fp16 parts (x = hi + lo, both exact to ~2^-22 relative), accumulating
//    one 32-element block in fp32; the block's fp16 scale d is applied to
//    that partial sum in fp32.  The result is accurate to fp32 level, like
//    the reference's dot_f32_quant (quant.c:103-155), which multiplies fp32
//    activations by d*q.
//  * K order inside a block is permuted (lane quad c owns bytes 8c..8c+7 of
//    each Q8_0 block), identically for weights and activations, so every
//    activation fragment is one 16-byte load.
//
// Every mbarrier wait is bounded: on expiry the kernel records an error in
// a device flag (read by the host) and leaves without touching the chunk.
#include "common.cuh"
#include "kernels.h"

#include <cuda_fp16.h>

namespace moe {

constexpr int kMmaWarps = 8;                 // consumer warps per CTA

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // bounded mbarrier waits: 2 s

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
	return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
	asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
		     : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
	asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async()
{
	asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
	asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
		     "r"(bytes)
		     : "memory");
}

// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or ~100 us pass, so waiting warps do not steal issue slots
// from the warps that are computing
__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
	asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
	uint32_t ok;
	asm volatile(
		"{\n\t.reg .pred p;\n\t"
		"mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 100000;\n\t"
		"selp.u32 %0, 1, 0, p;\n\t}"
		: "=r"(ok)
		: "r"(smem_addr(bar)), "r"(parity)
		: "memory");
	return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns()
{
	uint64_t t;
	asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
	return t;
}

// bounded wait; false when kWaitLimitNs of wall time passed
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity)
{
	if (mbar_try_wait(bar, parity))
		return true;
	const uint64_t t0 = global_ns();
	for (;;) {
		if (mbar_try_wait(bar, parity))
			return true;
		if (global_ns() - t0 > kWaitLimitNs)
			return false;
	}
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
	asm volatile(
		"cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
		::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
		: "memory");
}

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
					  uint32_t b1)
{
	asm volatile(
		"mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
		"{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
		: "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
		: "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// two int8 codes (low byte first) -> half2 of the exact integers
__device__ __forceinline__ uint32_t i8x2_to_h2(uint32_t w)
{
	const uint32_t biased = __byte_perm(w ^ 0x8080u, 0x64646464u, 0x4140);  // 1024 + q + 128
	const __half2 h = __hsub2(*reinterpret_cast<const __half2 *>(&biased),
				  __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));
	return *reinterpret_cast<const uint32_t *>(&h);
}

// nibbles (bits 0-3 and 16-19 of w) -> half2 of (nib - 8)
__device__ __forceinline__ uint32_t u4x2_to_h2(uint32_t w)
{
	const uint32_t biased = (w & 0x000F000Fu) | 0x64006400u;  // 1024 + nib
	const __half2 h = __hsub2(*reinterpret_cast<const __half2 *>(&biased),
				  __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408)));
	return *reinterpret_cast<const uint32_t *>(&h);
}

__device__ __forceinline__ uint16_t lds_u16(const uint8_t *p)
{
	return *reinterpret_cast<const uint16_t *>(p);
}

// A fragments (two k16 steps) of one 32-element block for rows g and g+8.
// Q8_0 (34-byte block, codes at +2): lane quad c owns codes 8c..8c+7:
//   step 0 = codes (8c,8c+1) | (8c+2,8c+3), step 1 = (8c+4,8c+5) | (8c+6,8c+7).
// Q4_0 (18-byte block, byte j = code j low nibble, code j+16 high nibble):
//   lane quad c owns bytes 4c..4c+3 and takes, per u32 of those bytes,
//   pairs (b0,b2) low, (b0,b2) high, (b1,b3) low, (b1,b3) high nibbles.
template <int QT>
__device__ __forceinline__ void load_a(const uint8_t *rg, const uint8_t *rg8, int c,
				       uint32_t (&a0)[4], uint32_t (&a1)[4], float &dg, float &dg8)
{
	dg = half_bits_to_float(lds_u16(rg));
	dg8 = half_bits_to_float(lds_u16(rg8));
	if (QT == kQ8_0) {
		const uint8_t *pg = rg + 2 + 8 * c, *p8 = rg8 + 2 + 8 * c;
		a0[0] = i8x2_to_h2(lds_u16(pg + 0));
		a0[1] = i8x2_to_h2(lds_u16(p8 + 0));
		a0[2] = i8x2_to_h2(lds_u16(pg + 2));
		a0[3] = i8x2_to_h2(lds_u16(p8 + 2));
		a1[0] = i8x2_to_h2(lds_u16(pg + 4));
		a1[1] = i8x2_to_h2(lds_u16(p8 + 4));
		a1[2] = i8x2_to_h2(lds_u16(pg + 6));
		a1[3] = i8x2_to_h2(lds_u16(p8 + 6));
	} else {
		const uint8_t *pg = rg + 2 + 4 * c, *p8 = rg8 + 2 + 4 * c;
		const uint32_t wg = (uint32_t)lds_u16(pg) | ((uint32_t)lds_u16(pg + 2) << 16);
		const uint32_t w8 = (uint32_t)lds_u16(p8) | ((uint32_t)lds_u16(p8 + 2) << 16);
		// wg bytes: b0 b1 b2 b3 -> (b0,b2) = bits 0-7 / 16-23, (b1,b3) = bits 8-15 / 24-31
		a0[0] = u4x2_to_h2(wg);          // low nibbles of b0, b2
		a0[1] = u4x2_to_h2(w8);
		a0[2] = u4x2_to_h2(wg >> 4);     // high nibbles of b0, b2
		a0[3] = u4x2_to_h2(w8 >> 4);
		a1[0] = u4x2_to_h2(wg >> 8);     // low nibbles of b1, b3
		a1[1] = u4x2_to_h2(w8 >> 8);
		a1[2] = u4x2_to_h2(wg >> 12);    // high nibbles of b1, b3
		a1[3] = u4x2_to_h2(w8 >> 12);
	}
}

// Q4_0 activation order: slot k = 8c + j of a 32-element block holds element
// [4c, 4c+2, 16+4c, 16+4c+2, 4c+1, 4c+3, 16+4c+1, 16+4c+3][j], matching the
// nibble pairs load_a<Q4_0> builds.  q4_slot maps an element to its slot.
__host__ __device__ __forceinline__ int q4_slot(int r)
{
	const int m = r & 31, h16 = m >> 4, mm = m & 15;
	const int c = mm >> 2, odd = mm & 1, two = (mm >> 1) & 1;
	return (r & ~31) | (8 * c + (two | (h16 << 1) | (odd << 2)));
}

__host__ __device__ __forceinline__ int q4_src(int k)
{
	const int base = k & ~31, c = (k & 31) >> 3, j = k & 7;
	return base + 4 * c + 16 * ((j >> 1) & 1) + ((j >> 2) & 1) + 2 * (j & 1);
}

// ---------------------------------------------------------------- kernel
// Warp-specialised CTA, one per SM: warps 0-7 do the math, warp 8 is the
// TMA producer, warps 9-10 run the epilogue.
//
// Work item = (active expert, 16-row tile): for DUAL, gate rows r0..r0+7
// and the same up rows (MMA rows 0-7 and 8-15, so gate and up of a (row,
// token) meet in one accumulator set for SwiGLU); for the single matrix,
// rows r0..r0+15.  An item is processed in passes of 8 tokens.  Each CTA
// takes a contiguous range of items balanced by cost (passes), which every
// warp derives identically from the routing table, so consecutive items
// mostly share an expert and its activations.
//
// Producer: per (item, pass, column chunk) one pipeline stage holding the
// tile's 16 weight rows over KC <= 2048 columns as 16 contiguous row copies
// (2176 B for a Q8_0 row of 2048) -- long runs of consecutive bytes, which
// HBM serves far better than short pieces of many rows.
// Math warps split the stage's K range (warp w owns columns w*KC/8 ..) and
// keep the matching activation fragments of the pass's 8 tokens in
// registers; at the end of a pass each writes its partial sums into one of
// kRedBufs exchange buffers and moves on.
// Epilogue warps (alternating passes) add the 8 partials in warp order
// (deterministic), apply SwiGLU or the output permutation and store.
// All waits are bounded; a warp whose wait expires records the error and
// keeps walking its loops without waiting, so no warp is left blocked.
constexpr int kTokTile = 8;          // tokens per pass (one MMA n-tile)
constexpr int kMaxKC = 2048;         // columns per stage
constexpr int kRedBufs = 4;          // partial-sum exchange buffers
constexpr int kEpiWarps = 2;

template <int QT>
struct StageLayout {
	static constexpr int BB = QT == kQ8_0 ? Q8_0_BYTES : Q4_0_BYTES;
	static constexpr int RS = kMaxKC / QK * BB + 16;          // smem row stride (padded)
	static constexpr int BYTES = 16 * RS;                    // one stage
	static constexpr int RED = kRedBufs * kMmaWarps * 32 * 16;
	static constexpr int META = kRedBufs * 16;               // per buffer: r0, n, off, tg
	static constexpr int TAB = 4 * 256 * 4;                  // (e|n), off, cost prefix [257]
};

// cost-balanced contiguous item range of this CTA.  cost(item) = passes of
// its expert; tab[512 + a] = cost of the items of active experts < a.
__device__ __forceinline__ void item_range(const int32_t *tab, int n_active, int groups,
					   int &i0, int &i1)
{
	const int total = tab[512 + n_active];
	const int64_t c0 = (int64_t)total * blockIdx.x / gridDim.x;
	const int64_t c1 = (int64_t)total * (blockIdx.x + 1) / gridDim.x;
	// first item whose cumulative cost start is >= c (items of expert a cost p_a each)
	auto first_item = [&](int64_t c) {
		int a = 0;
		while (a < n_active && tab[512 + a + 1] <= c)
			a++;
		if (a == n_active)
			return n_active * groups;
		const int pa = (tab[a] >> 8) > 0 ? ((tab[a] >> 8) + kTokTile - 1) / kTokTile : 1;
		const int64_t k = (c - tab[512 + a] + pa - 1) / pa;   // items of expert a before c
		return a * groups + (int)(k < groups ? k : groups);
	};
	i0 = first_item(c0);
	i1 = first_item(c1);
}

template <int QT, bool DUAL, int STAGES, int WB>
__global__ void __launch_bounds__((kMmaWarps + 1 + kEpiWarps) * 32, 1)
expert_mma_kernel(MmaArgs a)
{
	// WB = blocks per math warp per stage (KC = 256*WB columns); the
	// launcher guarantees cols % KC == 0
	extern __shared__ __align__(128) uint8_t smem[];
	using SL = StageLayout<QT>;
	constexpr int BB = SL::BB, RS = SL::RS;
	constexpr int ROWS = DUAL ? 8 : 16;  // matrix rows per item
	constexpr int KC = WB * kMmaWarps * QK;
	constexpr int PRODUCER = kMmaWarps, EPI0 = kMmaWarps + 1;

	const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
	uint8_t *p = smem + STAGES * SL::BYTES;
	float4 *red = reinterpret_cast<float4 *>(p);                  // [kRedBufs][8][32]
	int32_t *meta = reinterpret_cast<int32_t *>(p + SL::RED);     // [kRedBufs][4]
	int32_t *tab = reinterpret_cast<int32_t *>(p + SL::RED + SL::META);
	uint64_t *full = reinterpret_cast<uint64_t *>(p + SL::RED + SL::META + SL::TAB);
	uint64_t *empty = full + STAGES;
	uint64_t *rfull = empty + STAGES;
	uint64_t *rempty = rfull + kRedBufs;
	if (threadIdx.x < STAGES) {
		mbar_init(&full[threadIdx.x], 1);
		mbar_init(&empty[threadIdx.x], kMmaWarps);
	}
	if (threadIdx.x < kRedBufs) {
		mbar_init(&rfull[threadIdx.x], kMmaWarps);
		mbar_init(&rempty[threadIdx.x], 1);
	}
	// routing tables of the active experts, read once per CTA:
	// tab[i] = expert | pair count << 8, tab[256+i] = its offset,
	// tab[512+i] = cost (passes) of all items of active experts < i
	const int n_active = *a.n_active;
	const int groups = (a.rows + ROWS - 1) / ROWS;
	for (int i = threadIdx.x; i < n_active; i += blockDim.x) {
		const int e = a.active[i];
		tab[i] = e | (a.counts[e] << 8);
		tab[256 + i] = a.offsets[e];
	}
	__syncthreads();
	if (threadIdx.x == 0) {
		int c = 0;
		for (int i = 0; i < n_active; i++) {
			tab[512 + i] = c;
			c += groups * (((tab[i] >> 8) + kTokTile - 1) / kTokTile);
		}
		tab[512 + n_active] = c;
	}
	fence_mbar_init();
	__syncthreads();

	const int cols = a.cols;
	const int64_t rb = (int64_t)(cols / QK) * BB;
	const int nch = cols / KC;                 // column chunks per row
	int i0, i1;
	item_range(tab, n_active, groups, i0, i1);

	if (warp == PRODUCER) {
		// ------------------------------------------------ producer warp
		uint32_t it = 0;
		bool failed = false;
		int ai = i0 / groups, r0 = (i0 % groups) * ROWS;
		for (int item = i0; item < i1; item++, r0 += ROWS) {
			if (r0 >= groups * ROWS) {
				r0 = 0;
				ai++;
			}
			const int e = tab[ai] & 255;
			const int n = tab[ai] >> 8;
			// lane l (< 16) copies tile row l
			const uint8_t *src = nullptr;
			if (lane < 16) {
				const int r = DUAL ? r0 + (lane & 7) : r0 + lane;
				const uint8_t *base = static_cast<const uint8_t *>(
					(DUAL && lane >= 8) ? a.w2[e] : a.w1[e]);
				src = base + (int64_t)min(r, a.rows - 1) * rb;
			}
			for (int tg = 0; tg < n; tg += kTokTile) {
				for (int ch = 0; ch < nch; ch++, it++) {
					const int st = it % STAGES;
					if (it >= STAGES && !failed &&
					    !__all_sync(0xffffffffu, mbar_wait(&empty[st], ((it / STAGES) - 1) & 1))) {
						failed = true;
						if (lane == 0)
							atomicExch(a.err, 2);
					}
					if (failed)
						continue;
					constexpr uint32_t cb = (uint32_t)(KC / QK * BB);  // bytes per row
					if (lane == 0)
						mbar_arrive_expect_tx(&full[st], 16 * cb);
					__syncwarp();
					if (lane < 16) {
						fence_proxy_async();
						bulk_g2s(smem + st * SL::BYTES + lane * RS,
							 src + (int64_t)ch * (KC / QK) * BB, cb, &full[st]);
					}
				}
			}
		}
		return;
	}

	if (warp >= EPI0) {
		// ------------------------------------------------ epilogue warps
		bool failed = false;
		uint32_t pass = 0;
		int ai = i0 / groups, r0 = (i0 % groups) * ROWS;
		for (int item = i0; item < i1; item++, r0 += ROWS) {
			if (r0 >= groups * ROWS) {
				r0 = 0;
				ai++;
			}
			const int n = tab[ai] >> 8, off = tab[256 + ai];
			for (int tg = 0; tg < n; tg += kTokTile, pass++) {
				if ((int)(pass % kEpiWarps) != warp - EPI0)
					continue;
				const int buf = pass % kRedBufs;
				if (!failed &&
				    !__all_sync(0xffffffffu, mbar_wait(&rfull[buf], (pass / kRedBufs) & 1))) {
					failed = true;
					if (lane == 0)
						atomicExch(a.err, 2);
				}
				if (!failed) {
					const float *rv = reinterpret_cast<const float *>(red + buf * kMmaWarps * 32);
					// DUAL: 64 outputs (lane l of the MMA layout, token slot j),
					// gate = value j and up = value 2+j of that lane; 2 per thread.
					// Single: 128 outputs (lane l, value i); 4 per thread.
#pragma unroll
					for (int q = 0; q < (DUAL ? 2 : 4); q++) {
						const int o = lane + 32 * q;
						const int l = DUAL ? o >> 1 : o >> 2;
						const int i = DUAL ? (o & 1) : (o & 3);
						float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
						for (int w = 0; w < kMmaWarps; w++) {
							s0 = __fadd_rn(s0, rv[(w * 32 + l) * 4 + i]);
							if (DUAL)
								s1 = __fadd_rn(s1, rv[(w * 32 + l) * 4 + 2 + i]);
						}
						const int gg = l >> 2, cc = l & 3;
						const int t = tg + 2 * cc + (i & 1);
						if (t >= n)
							continue;
						const int pos = off + t;
						if (DUAL) {
							const int r = r0 + gg;
							if (r < a.rows) {
								const float h = swiglu(s0, s1);
								const __half hh = __float2half_rn(h);
								const __half hl = __float2half_rn(__fsub_rn(h, __half2float(hh)));
								__half *o16 = a.out16 + (int64_t)pos * 2 * a.rows;
								const int slot_r = QT == kQ4_0 ? q4_slot(r) : r;
								o16[slot_r] = hh;
								o16[a.rows + slot_r] = hl;
							}
						} else {
							const int r = r0 + gg + 8 * (i >> 1);
							const int orow = a.out_perm ? a.perm[pos] : pos;
							if (r < a.rows)
								a.out[(int64_t)orow * a.rows + r] = s0;
						}
					}
				}
				__syncwarp();
				if (lane == 0)
					mbar_arrive(&rempty[buf]);
			}
		}
		return;
	}

	// ---------------------------------------------------- math warps
	const int g = lane >> 2, c = lane & 3;
	bool failed = false;
	uint4 xh[WB], xl[WB];
	int x_e = -1, x_tg = -1, x_ch = -1;  // key of the fragments in registers
	uint32_t it = 0, pass = 0;
	int ai = i0 / groups, r0 = (i0 % groups) * ROWS;
	for (int item = i0; item < i1; item++, r0 += ROWS) {
		if (r0 >= groups * ROWS) {
			r0 = 0;
			ai++;
		}
		const int e = tab[ai] & 255;
		const int n = tab[ai] >> 8, off = tab[256 + ai];
		for (int tg = 0; tg < n; tg += kTokTile, pass++) {
			float acc[4] = {0.f, 0.f, 0.f, 0.f};
			for (int ch = 0; ch < nch; ch++, it++) {
				const int kb0 = ch * (KC / QK) + warp * WB;  // first block (row-global)
				if (e != x_e || tg != x_tg || ch != x_ch) {
					// token tg+g's activations for this warp's blocks; columns of
					// tokens past n read the segment's first token (never stored)
					const int t = tg + g < n ? tg + g : 0;
					const int pos = off + t;
					const int row = a.in_perm ? a.perm[pos] / a.K : pos;
					const __half *px = a.in16 + (int64_t)row * 2 * cols + 8 * c;
#pragma unroll
					for (int b = 0; b < WB; b++) {
						xh[b] = __ldg(reinterpret_cast<const uint4 *>(px + (kb0 + b) * QK));
						xl[b] = __ldg(reinterpret_cast<const uint4 *>(px + cols + (kb0 + b) * QK));
					}
					x_e = e;
					x_tg = tg;
					x_ch = ch;
				}
				const int st = it % STAGES;
				if (!failed &&
				    !__all_sync(0xffffffffu, mbar_wait(&full[st], (it / STAGES) & 1))) {
					failed = true;
					if (lane == 0)
						atomicExch(a.err, 2);
				}
				if (!failed) {
					const uint8_t *wt = smem + st * SL::BYTES + (warp * WB) * BB;
#pragma unroll
					for (int b = 0; b < WB; b++) {
						uint32_t A0[4], A1[4];
						float d0, d1;
						load_a<QT>(wt + g * RS + b * BB, wt + (g + 8) * RS + b * BB, c, A0,
							   A1, d0, d1);
						float t0[4] = {0.f, 0.f, 0.f, 0.f}, t1[4] = {0.f, 0.f, 0.f, 0.f};
						mma_16816(t0, A0, xh[b].x, xh[b].y);
						mma_16816(t1, A1, xh[b].z, xh[b].w);
						mma_16816(t0, A0, xl[b].x, xl[b].y);
						mma_16816(t1, A1, xl[b].z, xl[b].w);
						acc[0] = __fmaf_rn(d0, __fadd_rn(t0[0], t1[0]), acc[0]);
						acc[1] = __fmaf_rn(d0, __fadd_rn(t0[1], t1[1]), acc[1]);
						acc[2] = __fmaf_rn(d1, __fadd_rn(t0[2], t1[2]), acc[2]);
						acc[3] = __fmaf_rn(d1, __fadd_rn(t0[3], t1[3]), acc[3]);
					}
				}
				__syncwarp();
				if (lane == 0)
					mbar_arrive(&empty[st]);
			}
			// hand the partial sums to the epilogue warps
			const int buf = pass % kRedBufs;
			if (pass >= kRedBufs && !failed &&
			    !__all_sync(0xffffffffu, mbar_wait(&rempty[buf], ((pass / kRedBufs) - 1) & 1))) {
				failed = true;
				if (lane == 0)
					atomicExch(a.err, 2);
			}
			red[(buf * kMmaWarps + warp) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
			__syncwarp();
			if (lane == 0)
				mbar_arrive(&rfull[buf]);
		}
	}
}

// ---------------------------------------------------------------- x -> fp16 hi/lo
// out[r][0][k] = fp16(x), out[r][1][k] = fp16(x - hi).  For Q4_0 weights the
// 32 elements of each block are stored in the order the Q4_0 fragments use.
__global__ void split_f16_kernel(const float *__restrict__ x, int64_t rows, int cols, int q4,
				 __half *__restrict__ out)
{
	const int64_t total = rows * cols;
	for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
	     i += (int64_t)gridDim.x * blockDim.x) {
		const int64_t r = i / cols;
		const int k = (int)(i - r * cols);
		const int src = q4 ? q4_src(k) : k;
		const float v = x[r * cols + src];
		const __half h = __float2half_rn(v);
		out[r * 2 * cols + k] = h;
		out[r * 2 * cols + cols + k] = __float2half_rn(__fsub_rn(v, __half2float(h)));
	}
}

cudaError_t launch_split_f16(const float *x, int64_t rows, int cols, int qtype, __half *out,
			     cudaStream_t st)
{
	const int64_t total = rows * cols;
	if (total == 0)
		return cudaSuccess;
	int64_t blocks = (total + 255) / 256;
	if (blocks > 148 * 32)
		blocks = 148 * 32;
	split_f16_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, rows, cols, qtype == kQ4_0, out);
	return cudaGetLastError();
}

template <int QT, bool DUAL, int STAGES, int WB>
static cudaError_t launch_t(const MmaArgs &a, cudaStream_t st)
{
	using SL = StageLayout<QT>;
	const size_t smem = (size_t)STAGES * SL::BYTES + SL::RED + SL::META + SL::TAB +
			    (2 * STAGES + 2 * kRedBufs) * 8;
	auto fn = expert_mma_kernel<QT, DUAL, STAGES, WB>;
	constexpr int threads = (kMmaWarps + 1 + kEpiWarps) * 32;
	cudaError_t e = ensure_smem(fn, smem);
	if (e != cudaSuccess)
		return e;
	static int per_sm = 0;  // occupancy of this instantiation (fixed)
	if (!per_sm) {
		e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem);
		if (e != cudaSuccess)
			return e;
		if (per_sm < 1) {
			per_sm = 0;
			return cudaErrorInvalidConfiguration;
		}
	}
	const int sms = sm_count();
	int64_t grid = (int64_t)sms * per_sm;
	const int rows_per_item = DUAL ? 8 : 16;
	const int64_t max_items = (int64_t)a.n_local * ((a.rows + rows_per_item - 1) / rows_per_item);
	if (grid > max_items)
		grid = max_items;
	fn<<<(unsigned)grid, threads, smem, st>>>(a);
	return cudaGetLastError();
}

// blocks per consumer warp per stage: 8 (2048-column stages) when cols is a
// multiple of 2048, else cols/256 if that is 1, 2 or 4 (one stage per row)
static int pick_wb(int cols)
{
	if (cols % 2048 == 0)
		return 8;
	if (cols == 1024 || cols == 512 || cols == 256)
		return cols / 256;
	return 0;
}

bool expert_mma_supported(int qtype, int cols)
{
	return (qtype == kQ8_0 || qtype == kQ4_0) && pick_wb(cols) > 0;
}

template <int QT, bool DUAL, int S>
static cudaError_t launch_wb(const MmaArgs &a, cudaStream_t st)
{
	switch (pick_wb(a.cols)) {
	case 8: return launch_t<QT, DUAL, S, 8>(a, st);
	case 4: return launch_t<QT, DUAL, S, 4>(a, st);
	case 2: return launch_t<QT, DUAL, S, 2>(a, st);
	case 1: return launch_t<QT, DUAL, S, 1>(a, st);
	default: return cudaErrorInvalidValue;
	}
}

cudaError_t launch_expert_mma(const MmaArgs &a, cudaStream_t st)
{
	if (a.n_local <= 0 || a.rows <= 0)
		return cudaSuccess;
	if (!expert_mma_supported(a.qtype, a.cols))
		return cudaErrorInvalidValue;
	// one CTA per SM: 8 math warps (2 per scheduler) keep up with HBM,
	// and the whole shared memory goes to a deep copy pipeline
	if (a.qtype == kQ8_0)
		return a.dual ? launch_wb<kQ8_0, true, 5>(a, st) : launch_wb<kQ8_0, false, 5>(a, st);
	return a.dual ? launch_wb<kQ4_0, true, 9>(a, st) : launch_wb<kQ4_0, false, 9>(a, st);
}

}  // namespace moe
