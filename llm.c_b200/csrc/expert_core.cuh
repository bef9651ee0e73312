// expert_core.cuh — the warp-specialised grouped expert pipeline (decode),
// shared by the stand-alone expert kernel (expert_mma.cu) and the fused
// decode-layer kernel (decode.cu).
//
// Work: for every expert e with n_e routed (token, slot) pairs, stream the
// expert's Q8_0/Q4_0 weight rows from HBM once and multiply them with the
// n_e activation rows (fused SwiGLU for gate/up, plain for down).  This is
// the memory-bound regime (n_e is ~1-32 at decode), so the pipeline is built
// around moving bytes:
//
//  * One producer warp copies whole tile rows (16 rows x up to 2048 columns,
//    2176 contiguous bytes per Q8_0 row) into a ring of shared-memory stages
//    with cp.async.bulk, completing on per-stage mbarriers.  Long runs of
//    consecutive bytes keep HBM at its copy bandwidth.
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
//  * Eight math warps split each stage's K range and hand fp32 partial sums
//    to two epilogue warps through a 4-deep ring of exchange buffers; the
//    epilogue adds them in warp order (deterministic), applies SwiGLU or the
//    output permutation and stores.
//
// Every mbarrier wait is bounded: on expiry the waiting warp records an
// error in a device flag (read by the host) and keeps walking its loops
// without waiting, so no warp is left blocked and the kernel ends.
#pragma once

#include "common.cuh"

#include <cuda_fp16.h>

#include <type_traits>

namespace moe {

constexpr int kMmaWarps = 8;                 // math warps per CTA
constexpr int kTokTile = 8;                  // tokens per pass (one MMA n-tile)
// An expert with more than 8 tokens streams its rows once per token tile:
// the items of a CTA's segment are walked in chunks of this many, tile by
// tile, so that the rows of the second and later tiles (the chunk's ~560 KB,
// ~80 MB over the grid) are still in L2.  Activations are reloaded once per
// chunk and tile instead of once per segment and tile.
constexpr int kChunkItems = 16;
constexpr int kMaxKC = 2048;                 // columns per stage
constexpr int kRedBufs = 4;                  // partial-sum exchange buffers
constexpr int kEpiWarps = 2;
constexpr int kProducerWarp = kMmaWarps;
constexpr int kEpiWarp0 = kMmaWarps + 1;
constexpr int kCoreThreads = (kMmaWarps + 1 + kEpiWarps) * 32;
constexpr int kEpiStage = 8 * 32;  // floats of staging per epilogue warp
constexpr int kMaxActive = 256;              // experts per layer (routing tables)

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // bounded waits: 2 s

// f(std::integral_constant<int, i>) for i = 0 .. N-1, unrolled at compile time
template <int I, int N, typename F>
__device__ __forceinline__ void static_for_impl(F &&f)
{
	if constexpr (I < N) {
		f(std::integral_constant<int, I>{});
		static_for_impl<I + 1, N>(f);
	}
}

template <int N, typename F>
__device__ __forceinline__ void static_for(F &&f)
{
	static_for_impl<0, N>(f);
}

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

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
	asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or ~100 us pass, so waiting warps do not steal issue slots
// from the warps that are computing
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
// nibble pairs load_a<Q4_0> builds.  q4_slot maps an element to its slot,
// q4_src a slot to its element.
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

// ---------------------------------------------------------------- biased fragments
// Used when a warp's blocks sit at known positions mod 4 in the stage row
// (WB % 4 == 0), so every code byte is read with aligned 32/64-bit loads.
// The loads build fp16 values code + BIAS with bit operations only (exact:
// 1152 + q for Q8_0 from 0x6400 | (q ^ 0x80), 1024 + nib = (nib - 8) + 1032
// for Q4_0); unbias2 then subtracts BIAS exactly, one instruction per pair.
// (Feeding the biased values to the MMA and removing BIAS * (block sum of
// the activations) afterwards is cheaper but cancels ~10 bits in fp32.)
template <int QT>
struct Bias {
	static constexpr unsigned short half = QT == kQ8_0 ? 0x6480 : 0x6408;  // fp16 1152 / 1032
};

// biased fp16 pair (BIAS + c0, BIAS + c1) -> the exact codes (c0, c1): the
// subtraction is exact (both are integers below 2048)
template <int QT>
__device__ __forceinline__ uint32_t unbias2(uint32_t a)
{
	const __half2 b = __halves2half2(__ushort_as_half(Bias<QT>::half), __ushort_as_half(Bias<QT>::half));
	const __half2 r = __hsub2(*reinterpret_cast<const __half2 *>(&a), b);
	return *reinterpret_cast<const uint32_t *>(&r);
}

// the 8 code bytes of a Q8_0 block at position JM (mod 4) of its row,
// p = block + 2 + 8c: rows are 8-byte aligned and blocks 34 bytes long, so
// p is 2, 4, 6 or 0 (mod 8) for JM = 0, 1, 2, 3
template <int JM>
__device__ __forceinline__ void lds_q8_codes(const uint8_t *p, uint32_t &w0, uint32_t &w1)
{
	if (JM == 3) {
		const uint2 v = *reinterpret_cast<const uint2 *>(p);
		w0 = v.x;
		w1 = v.y;
	} else if (JM == 1) {
		w0 = *reinterpret_cast<const uint32_t *>(p);
		w1 = *reinterpret_cast<const uint32_t *>(p + 4);
	} else if (JM == 0) {
		const uint2 v = *reinterpret_cast<const uint2 *>(p - 2);
		const uint32_t w2 = *reinterpret_cast<const uint32_t *>(p + 6);
		w0 = __byte_perm(v.x, v.y, 0x5432);
		w1 = __byte_perm(v.y, w2, 0x5432);
	} else {
		const uint32_t v0 = *reinterpret_cast<const uint32_t *>(p - 2);
		const uint2 v = *reinterpret_cast<const uint2 *>(p + 2);
		w0 = __byte_perm(v0, v.x, 0x5432);
		w1 = __byte_perm(v.x, v.y, 0x5432);
	}
}

// the 4 code bytes of a Q4_0 block at position JM (mod 2), p = block + 2 + 4c
template <int JM>
__device__ __forceinline__ uint32_t lds_q4_codes(const uint8_t *p)
{
	if (JM == 1)
		return *reinterpret_cast<const uint32_t *>(p);
	return __byte_perm(*reinterpret_cast<const uint32_t *>(p - 2),
			   *reinterpret_cast<const uint32_t *>(p + 2), 0x5432);
}

// biased A fragments (same k slots as load_a) of block J for rows g, g+8
template <int QT, int J>
__device__ __forceinline__ void load_a_biased(const uint8_t *rg, const uint8_t *rg8, int c,
					      uint32_t (&a0)[4], uint32_t (&a1)[4], float &dg,
					      float &dg8)
{
	dg = half_bits_to_float(lds_u16(rg));
	dg8 = half_bits_to_float(lds_u16(rg8));
	if (QT == kQ8_0) {
		constexpr uint32_t E = 0x64646464u;
		uint32_t g0, g1, h0, h1;
		lds_q8_codes<J % 4>(rg + 2 + 8 * c, g0, g1);
		lds_q8_codes<J % 4>(rg8 + 2 + 8 * c, h0, h1);
		g0 ^= 0x80808080u;
		g1 ^= 0x80808080u;
		h0 ^= 0x80808080u;
		h1 ^= 0x80808080u;
		a0[0] = __byte_perm(g0, E, 0x4140);  // codes 8c, 8c+1
		a0[1] = __byte_perm(h0, E, 0x4140);
		a0[2] = __byte_perm(g0, E, 0x4342);  // codes 8c+2, 8c+3
		a0[3] = __byte_perm(h0, E, 0x4342);
		a1[0] = __byte_perm(g1, E, 0x4140);  // codes 8c+4, 8c+5
		a1[1] = __byte_perm(h1, E, 0x4140);
		a1[2] = __byte_perm(g1, E, 0x4342);  // codes 8c+6, 8c+7
		a1[3] = __byte_perm(h1, E, 0x4342);
	} else {
		const uint32_t wg = lds_q4_codes<J % 2>(rg + 2 + 4 * c);
		const uint32_t w8 = lds_q4_codes<J % 2>(rg8 + 2 + 4 * c);
		constexpr uint32_t M = 0x000F000Fu, E = 0x64006400u;
		a0[0] = (wg & M) | E;          // low nibbles of b0, b2
		a0[1] = (w8 & M) | E;
		a0[2] = ((wg >> 4) & M) | E;   // high nibbles of b0, b2
		a0[3] = ((w8 >> 4) & M) | E;
		a1[0] = ((wg >> 8) & M) | E;   // low nibbles of b1, b3
		a1[1] = ((w8 >> 8) & M) | E;
		a1[2] = ((wg >> 12) & M) | E;  // high nibbles of b1, b3
		a1[3] = ((w8 >> 12) & M) | E;
	}
}

// ---------------------------------------------------------------- layout
template <int QT>
struct StageLayout {
	static constexpr int BB = QT == kQ8_0 ? Q8_0_BYTES : Q4_0_BYTES;
	static constexpr int RS = kMaxKC / QK * BB + 16;          // smem row stride (padded)
	static constexpr int BYTES = 16 * RS;                    // one stage
	static constexpr int RED = kRedBufs * kMmaWarps * 32 * 16;
	static constexpr int EPI = kEpiWarps * kEpiStage * 4;  // epilogue staging tiles
	// two 1024-column rows share one row slot (items of two m-tiles): rows
	// 2j and 2j + 1 of the item, adjacent as in HBM, so one copy of 2 rows
	// fills the slot; the second starts here (16-byte aligned)
	static constexpr int HALF = 1024 / QK * BB;
	static_assert(HALF + 1024 / QK * BB <= RS && HALF % 16 == 0, "two half rows per slot");
};

// One grouped matrix pass (gate/up with SwiGLU, or down).
//
// Work item = (active expert, 16-row tile): for DUAL, gate rows r0..r0+7
// and the same up rows (MMA rows 0-7 and 8-15, so gate and up of a (row,
// token) meet in one accumulator set for SwiGLU); for the single matrix,
// rows r0..r0+15.  An item is processed in passes of 8 tokens.  Each CTA
// takes a contiguous range of items balanced by cost (passes), which every
// warp derives identically from the routing table.  Within the range, the
// items of one expert (a segment) are walked token tile by token tile, so
// the math warps load each tile's activations once per segment; the weights
// of a second token tile come back from L2.
//   in  row of position pos: in_perm  ? in16[perm[pos] / K] : in16[pos]
//   out row of position pos: out_perm ? out[perm[pos]]      : out[pos]
struct Phase {
	const void *const *w1;   // device table [experts] of weight pointers
	const void *const *w2;   // DUAL: the up matrices
	int rows, cols, K;
	const int32_t *en;       // [n_active] expert | pair count << 8
	const int32_t *off;      // [n_active] first position of the expert
	const int32_t *pre;      // [n_active + 1] cost prefix (passes x tiles)
	int n_active;
	const int32_t *perm;     // [pairs] pair of each position
	int in_perm, out_perm;
	const __half *in16;      // [*, 2, cols] fp16 hi/lo
	__half *out16;           // DUAL: [*, 2, rows] fp16 hi/lo
	float *out;              // single: [*, rows] fp32
	int32_t *err;            // set to 2 when a bounded wait expires
	const float *wdiv;       // single, optional: store y / (1 / wdiv[out row])
	float *const *peers;     // single, optional: the same rows also go to these
	int npeers;              // buffers (other GPUs' memory, expert parallelism)
	// single, token-sharded expert parallelism: out row `orow` belongs to
	// rank orow / shard_pairs and goes to peers[that rank] at row
	// orow % shard_pairs (peers then holds every rank's buffer, own one
	// included, and `out` is unused)
	int shard_pairs;
};

struct Bars {
	uint64_t *full, *empty;      // [STAGES]
	uint64_t *rfull, *rempty;    // [kRedBufs]
};

// per-thread pipeline position, carried across consecutive phases
struct Pipe {
	uint32_t it = 0;    // stage sequence number
	uint32_t pass = 0;  // partial-sum exchange sequence number
	bool failed = false;
};

__device__ __forceinline__ int passes_of(int en) { return ((en >> 8) + kTokTile - 1) / kTokTile; }

// cost prefix of the active experts' items: pre[a] = cost of the items of
// active experts < a, cost(item) = passes of its expert
__device__ __forceinline__ void build_prefix(const int32_t *en, int n_active, int groups,
					     int32_t *pre)
{
	int c = 0;
	for (int i = 0; i < n_active; i++) {
		pre[i] = c;
		c += groups * passes_of(en[i]);
	}
	pre[n_active] = c;
}

// the same prefix computed by one whole warp (inclusive scan by shuffles)
__device__ __forceinline__ void build_prefix_warp(const int32_t *en, int n_active, int groups,
						  int32_t *pre)
{
	const int lane = threadIdx.x % 32;
	int carry = 0;
	for (int base = 0; base < n_active; base += 32) {
		const int i = base + lane;
		const int c = i < n_active ? groups * passes_of(en[i]) : 0;
		int incl = c;
#pragma unroll
		for (int o = 1; o < 32; o <<= 1) {
			const int u = __shfl_up_sync(0xffffffffu, incl, o);
			if (lane >= o)
				incl += u;
		}
		if (i < n_active)
			pre[i] = carry + incl - c;
		carry += __shfl_sync(0xffffffffu, incl, 31);
	}
	if (lane == 0)
		pre[n_active] = carry;
	__syncwarp();
}

// cost-balanced contiguous item range of this CTA
__device__ __forceinline__ void item_range(const int32_t *en, const int32_t *pre, int n_active,
					   int groups, int &i0, int &i1)
{
	const int total = pre[n_active];
	const int64_t c0 = (int64_t)total * blockIdx.x / gridDim.x;
	const int64_t c1 = (int64_t)total * (blockIdx.x + 1) / gridDim.x;
	// first item whose cumulative cost start is >= c (items of expert a cost p_a each)
	auto first_item = [&](int64_t c) {
		int a = 0;
		while (a < n_active && pre[a + 1] <= c)
			a++;
		if (a == n_active)
			return n_active * groups;
		const int pa = passes_of(en[a]) > 0 ? passes_of(en[a]) : 1;
		const int64_t k = (c - pre[a] + pa - 1) / pa;   // items of expert a before c
		return a * groups + (int)(k < groups ? k : groups);
	};
	i0 = first_item(c0);
	i1 = first_item(c1);
}

// ---------------------------------------------------------------- producer
template <int QT, bool DUAL, int STAGES, int WB, int MT = 1>
__device__ void core_producer(const Phase &ph, uint8_t *stages, const Bars &b, Pipe &p, int lane)
{
	using SL = StageLayout<QT>;
	constexpr int BB = SL::BB, RS = SL::RS;
	constexpr int ROWS = DUAL ? 8 : 16 * MT;
	constexpr int COPY_ROWS = DUAL ? 16 : 16 * MT;  // weight rows per stage
	constexpr int KC = WB * (kMmaWarps / MT) * QK;
	static_assert(MT == 1 || (MT == 2 && !DUAL && KC == 1024), "two m-tiles: 1024-column rows");
	constexpr uint32_t cb = (uint32_t)(KC / QK * BB);  // bytes per row and stage
	const int groups = (ph.rows + ROWS - 1) / ROWS;
	const int nch = ph.cols / KC;
	const int64_t rb = (int64_t)(ph.cols / QK) * BB;
	int i0, i1;
	item_range(ph.en, ph.pre, ph.n_active, groups, i0, i1);
	for (int seg = i0; seg < i1;) {
		const int ai = seg / groups, seg_end = min(i1, (ai + 1) * groups);
		const int e = ph.en[ai] & 255;
		const int n = ph.en[ai] >> 8;
		const uint8_t *base = static_cast<const uint8_t *>(
			(DUAL && lane >= 8) ? ph.w2[e] : ph.w1[e]);
		for (int c0 = seg; c0 < seg_end; c0 += kChunkItems)
		for (int tg = 0; tg < n; tg += kTokTile)
		for (int item = c0; item < min(seg_end, c0 + kChunkItems); item++) {
			const int r0 = (item - ai * groups) * ROWS;
			// lane l (< COPY_ROWS) copies tile row l; two m-tiles: m-tile m's
			// row j is item row 2j + m, and lane j < 16 copies rows 2j, 2j + 1
			// with one request when both exist (copy requests, not bytes,
			// bound the rate of 1 KB rows)
			const bool pair = MT == 2 && r0 + 2 * (lane & 15) + 1 < ph.rows;
			const int r = DUAL ? r0 + (lane & 7) : MT == 2 ? r0 + 2 * (lane & 15) + (lane >> 4) : r0 + lane;
			const uint8_t *src = base + (int64_t)min(r, ph.rows - 1) * rb;
			for (int ch = 0; ch < nch; ch++, p.it++) {
				const int st = p.it % STAGES;
				if (p.it >= STAGES && !p.failed &&
				    !__all_sync(0xffffffffu, mbar_wait(&b.empty[st], ((p.it / STAGES) - 1) & 1))) {
					p.failed = true;
					if (lane == 0)
						atomicExch(ph.err, 2);
				}
				if (p.failed)
					continue;
				if (lane == 0)
					mbar_arrive_expect_tx(&b.full[st], COPY_ROWS * cb);
				__syncwarp();
				// m-tile 1 of a two-tile item goes to the second half of the slot
				const int dst = MT == 2 ? (lane & 15) * RS + (lane >> 4) * SL::HALF : lane * RS;
				if (MT == 2 && pair) {
					if (lane < 16) {
						fence_proxy_async();
						bulk_g2s(stages + st * SL::BYTES + dst, src + (int64_t)ch * (KC / QK) * BB,
							 2 * cb, &b.full[st]);
					}
				} else if (lane < COPY_ROWS) {
					fence_proxy_async();
					bulk_g2s(stages + st * SL::BYTES + dst, src + (int64_t)ch * (KC / QK) * BB, cb,
						 &b.full[st]);
				}
			}
		}
		seg = seg_end;
	}
}

// ---------------------------------------------------------------- epilogue
// stg: this warp's staging tile (kEpiStage floats): the sums are written
// there in MMA order and leave as contiguous 16-byte stores per token row.
template <int QT, bool DUAL, int MT = 1>
__device__ void core_epilogue(const Phase &ph, const float4 *red, float *stg, const Bars &b,
			      Pipe &p, int epi, int lane)
{
	constexpr int ROWS = DUAL ? 8 : 16 * MT;
	constexpr int KW = kMmaWarps / MT;  // warps (K slices) per m-tile
	const int groups = (ph.rows + ROWS - 1) / ROWS;
	int i0, i1;
	item_range(ph.en, ph.pre, ph.n_active, groups, i0, i1);
	for (int seg = i0; seg < i1;) {
		const int ai = seg / groups, seg_end = min(i1, (ai + 1) * groups);
		const int n = ph.en[ai] >> 8, off = ph.off[ai];
		for (int c0 = seg; c0 < seg_end; c0 += kChunkItems)
		for (int tg = 0; tg < n; tg += kTokTile)
		for (int item = c0; item < min(seg_end, c0 + kChunkItems); item++, p.pass++) {
			const int r0 = (item - ai * groups) * ROWS;
			if ((int)(p.pass % kEpiWarps) != epi)
				continue;
			const int buf = p.pass % kRedBufs;
			if (!p.failed &&
			    !__all_sync(0xffffffffu, mbar_wait(&b.rfull[buf], (p.pass / kRedBufs) & 1))) {
				p.failed = true;
				if (lane == 0)
					atomicExch(ph.err, 2);
			}
			if (!p.failed) {
				const float *rv = reinterpret_cast<const float *>(red + buf * kMmaWarps * 32);
				// DUAL: 64 outputs (lane l of the MMA layout, token slot j),
				// gate = value j and up = value 2+j of that lane; 2 per thread.
				// Single: 128 outputs per m-tile (lane l, value i); 4 per thread
				// and m-tile, the K-slice partials added in warp order.
#pragma unroll
				for (int q = 0; q < (DUAL ? 2 : 4 * MT); q++) {
					const int o = lane + 32 * q;
					const int m = DUAL ? 0 : o >> 7;  // m-tile
					const int l = DUAL ? o >> 1 : (o & 127) >> 2;
					const int i = DUAL ? (o & 1) : (o & 3);
					float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
					for (int w = 0; w < KW; w++) {
						s0 = __fadd_rn(s0, rv[((m * KW + w) * 32 + l) * 4 + i]);
						if (DUAL)
							s1 = __fadd_rn(s1, rv[(w * 32 + l) * 4 + 2 + i]);
					}
					const int gg = l >> 2, cc = l & 3;
					const int tt = 2 * cc + (i & 1);  // token slot in the pass
					const int t = tg + tt;
					const int pos = off + (t < n ? t : 0);
					if (DUAL) {
						// h = silu(gate) * up, stored as fp16 hi + lo
						const float h = swiglu(s0, s1);
						const __half hh = __float2half_rn(h);
						const __half hl = __float2half_rn(__fsub_rn(h, __half2float(hh)));
						if (QT == kQ8_0) {
							__half *st16 = reinterpret_cast<__half *>(stg);
							st16[tt * 16 + gg] = hh;       // [token][hi 8 | lo 8]
							st16[tt * 16 + 8 + gg] = hl;
						} else if (t < n && r0 + gg < ph.rows) {
							const int r = r0 + gg;
							__half *o16 = ph.out16 + (int64_t)pos * 2 * ph.rows;
							o16[q4_slot(r)] = hh;
							o16[ph.rows + q4_slot(r)] = hl;
						}
					} else {
						// the combine's division (olmoe.c:397-404: y / (1 / w)),
						// done here where y is produced
						const int orow = ph.out_perm ? ph.perm[pos] : pos;
						const float v =
							ph.wdiv ? __fdiv_rn(s0, __fdiv_rn(1.0f, ph.wdiv[orow])) : s0;
						// [token][item row]; m-tile m's row j is item row 2j + m
						stg[tt * ROWS + (MT == 2 ? 2 * (gg + 8 * (i >> 1)) + m : gg + 8 * (i >> 1))] = v;
					}
				}
				__syncwarp();
				// rows of this item that exist, and whether 16-byte stores line up
				const int nr = min(ROWS, ph.rows - r0);
				if (DUAL && QT == kQ8_0) {
					// 8 tokens x (8 hi, 8 lo) halves: lane -> (token, hi|lo)
					if (lane < 16) {
						const int tt = lane >> 1, t = tg + tt;
						if (t < n) {
							const __half *src = reinterpret_cast<const __half *>(stg) + lane * 8;
							__half *o16 = ph.out16 + (int64_t)(off + t) * 2 * ph.rows +
								      (lane & 1) * ph.rows + r0;
							if (nr == 8 && ph.rows % 8 == 0)
								*reinterpret_cast<uint4 *>(o16) =
									*reinterpret_cast<const uint4 *>(src);
							else
								for (int r = 0; r < nr; r++)
									o16[r] = src[r];
						}
					}
				} else if (!DUAL) {
					// 8 tokens x ROWS rows: lane -> (token, ROWS/4 consecutive rows)
					constexpr int PER = ROWS / 4;
					const int tt = lane >> 2, t = tg + tt;
					if (t < n) {
						const int pos = off + t;
						int orow = ph.out_perm ? ph.perm[pos] : pos;
						const int rr = (lane & 3) * PER;
						float *obase = ph.out;
						if (ph.shard_pairs) {
							const int owner = orow / ph.shard_pairs;
							obase = ph.peers[owner];
							orow -= owner * ph.shard_pairs;
						}
						float *dst = obase + (int64_t)orow * ph.rows + r0 + rr;
						const float *src = stg + tt * ROWS + rr;
						if (nr == ROWS && ph.rows % 4 == 0) {
#pragma unroll
							for (int v = 0; v < PER; v += 4)
								*reinterpret_cast<float4 *>(dst + v) =
									*reinterpret_cast<const float4 *>(src + v);
							// expert parallelism: every GPU gets the row, written
							// over NVLink while the next tiles are computed
							for (int q = 0; q < ph.npeers; q++) {
								float *pd = ph.peers[q] + (int64_t)orow * ph.rows + r0 + rr;
#pragma unroll
								for (int v = 0; v < PER; v += 4)
									*reinterpret_cast<float4 *>(pd + v) =
										*reinterpret_cast<const float4 *>(src + v);
							}
						} else {
							for (int v = 0; v < PER && rr + v < nr; v++) {
								dst[v] = src[v];
								for (int q = 0; q < ph.npeers; q++)
									ph.peers[q][(int64_t)orow * ph.rows + r0 + rr + v] = src[v];
							}
						}
					}
				}
			}
			__syncwarp();
			if (lane == 0)
				mbar_arrive(&b.rempty[buf]);
		}
		seg = seg_end;
	}
}

// ---------------------------------------------------------------- math warps
// COHERENT: the activations were written earlier in the same kernel by
// other CTAs, so they are read through L2 (ld.global.cg), not the
// read-only path.  PF: rows span several stages; as each block's activation
// fragments are used up, the same token tile's fragments of the next column
// chunk are loaded into them, so the next stage does not start with a round
// trip to L2 (a wrong guess, at a tile or segment change, is caught by the
// key check and reloaded).
template <int QT, bool DUAL, int STAGES, int WB, bool COHERENT, int MT = 1, bool PF = false>
__device__ void core_math(const Phase &ph, const uint8_t *stages, float4 *red,
			  const Bars &b, Pipe &p, int warp, int lane)
{
	constexpr bool FAST = WB % 4 == 0;  // biased fragments, aligned code loads
	using SL = StageLayout<QT>;
	constexpr int BB = SL::BB, RS = SL::RS;
	constexpr int ROWS = DUAL ? 8 : 16 * MT;
	constexpr int KW = kMmaWarps / MT;  // K slices; warp = (m-tile, K slice)
	constexpr int KC = WB * KW * QK;
	const int mt = warp / KW, kq = warp % KW;
	const int groups = (ph.rows + ROWS - 1) / ROWS;
	const int cols = ph.cols;
	const int nch = cols / KC;
	const int g = lane >> 2, c = lane & 3;
	uint4 xh[WB], xl[WB];
	int x_e = -1, x_tg = -1, x_ch = -1;  // key of the fragments in registers
	const __half *x_px = nullptr;        // their token row (hi part, lane quad c)
	int i0, i1;
	item_range(ph.en, ph.pre, ph.n_active, groups, i0, i1);
	for (int seg = i0; seg < i1;) {
		const int ai = seg / groups, seg_end = min(i1, (ai + 1) * groups);
		const int e = ph.en[ai] & 255;
		const int n = ph.en[ai] >> 8, off = ph.off[ai];
		for (int c0 = seg; c0 < seg_end; c0 += kChunkItems)
		for (int tg = 0; tg < n; tg += kTokTile)
		for (int item = c0; item < min(seg_end, c0 + kChunkItems); item++, p.pass++) {
			float acc[4] = {0.f, 0.f, 0.f, 0.f};
			for (int ch = 0; ch < nch; ch++, p.it++) {
				const int kb0 = ch * (KC / QK) + kq * WB;  // first block (row-global)
				if (e != x_e || tg != x_tg || ch != x_ch) {
					// token tg+g's activations for this warp's blocks; columns of
					// tokens past n read the segment's first token (never stored)
					const int t = tg + g < n ? tg + g : 0;
					const int pos = off + t;
					const int row = ph.in_perm ? ph.perm[pos] / ph.K : pos;
					const __half *px = ph.in16 + (int64_t)row * 2 * cols + 8 * c;
					x_px = px;
#pragma unroll
					for (int bq = 0; bq < WB; bq++) {
						const uint4 *ph_ = reinterpret_cast<const uint4 *>(px + (kb0 + bq) * QK);
						const uint4 *pl_ =
							reinterpret_cast<const uint4 *>(px + cols + (kb0 + bq) * QK);
						xh[bq] = COHERENT ? __ldcg(ph_) : __ldg(ph_);
						xl[bq] = COHERENT ? __ldcg(pl_) : __ldg(pl_);
					}
					x_e = e;
					x_tg = tg;
					x_ch = ch;
				}
				const int st = p.it % STAGES;
				if (!p.failed &&
				    !__all_sync(0xffffffffu, mbar_wait(&b.full[st], (p.it / STAGES) & 1))) {
					p.failed = true;
					if (lane == 0)
						atomicExch(ph.err, 2);
				}
				if (!p.failed) {
					const uint8_t *wt =
						stages + st * SL::BYTES + (kq * WB) * BB + (MT == 2 ? mt * SL::HALF : 0);
					const bool pf = PF && nch > 1;
					const int ch_n = ch + 1 < nch ? ch + 1 : 0;
					const __half *pf_src = x_px + (ch_n * (KC / QK) + kq * WB) * QK;
					if constexpr (FAST) {
						static_for<WB>([&](auto J) {
							constexpr int bq = decltype(J)::value;
							uint32_t A0[4], A1[4];
							float d0, d1;
							load_a_biased<QT, bq>(wt + g * RS + bq * BB, wt + (g + 8) * RS + bq * BB,
									      c, A0, A1, d0, d1);
							// exact codes: the products and the block sums stay
							// small, so fp32 keeps them to ~1e-7
#pragma unroll
							for (int j = 0; j < 4; j++) {
								A0[j] = unbias2<QT>(A0[j]);
								A1[j] = unbias2<QT>(A1[j]);
							}
							float t[4] = {0.f, 0.f, 0.f, 0.f};
							mma_16816(t, A0, xh[bq].x, xh[bq].y);
							mma_16816(t, A1, xh[bq].z, xh[bq].w);
							mma_16816(t, A0, xl[bq].x, xl[bq].y);
							mma_16816(t, A1, xl[bq].z, xl[bq].w);
							acc[0] = __fmaf_rn(d0, t[0], acc[0]);
							acc[1] = __fmaf_rn(d0, t[1], acc[1]);
							acc[2] = __fmaf_rn(d1, t[2], acc[2]);
							acc[3] = __fmaf_rn(d1, t[3], acc[3]);
							if (pf) {
								const uint4 *ph_ = reinterpret_cast<const uint4 *>(pf_src + bq * QK);
								const uint4 *pl_ = reinterpret_cast<const uint4 *>(pf_src + cols + bq * QK);
								xh[bq] = COHERENT ? __ldcg(ph_) : __ldg(ph_);
								xl[bq] = COHERENT ? __ldcg(pl_) : __ldg(pl_);
							}
						});
						if (pf)
							x_ch = ch_n;
					} else
#pragma unroll
					for (int bq = 0; bq < WB; bq++) {
						uint32_t A0[4], A1[4];
						float d0, d1;
						load_a<QT>(wt + g * RS + bq * BB, wt + (g + 8) * RS + bq * BB, c, A0,
							   A1, d0, d1);
						float t0[4] = {0.f, 0.f, 0.f, 0.f}, t1[4] = {0.f, 0.f, 0.f, 0.f};
						mma_16816(t0, A0, xh[bq].x, xh[bq].y);
						mma_16816(t1, A1, xh[bq].z, xh[bq].w);
						mma_16816(t0, A0, xl[bq].x, xl[bq].y);
						mma_16816(t1, A1, xl[bq].z, xl[bq].w);
						acc[0] = __fmaf_rn(d0, __fadd_rn(t0[0], t1[0]), acc[0]);
						acc[1] = __fmaf_rn(d0, __fadd_rn(t0[1], t1[1]), acc[1]);
						acc[2] = __fmaf_rn(d1, __fadd_rn(t0[2], t1[2]), acc[2]);
						acc[3] = __fmaf_rn(d1, __fadd_rn(t0[3], t1[3]), acc[3]);
					}
				}
				__syncwarp();
				if (lane == 0)
					mbar_arrive(&b.empty[st]);
			}
			// hand the partial sums to the epilogue warps
			const int buf = p.pass % kRedBufs;
			if (p.pass >= kRedBufs && !p.failed &&
			    !__all_sync(0xffffffffu, mbar_wait(&b.rempty[buf], ((p.pass / kRedBufs) - 1) & 1))) {
				p.failed = true;
				if (lane == 0)
					atomicExch(ph.err, 2);
			}
			red[(buf * kMmaWarps + warp) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
			__syncwarp();
			if (lane == 0)
				mbar_arrive(&b.rfull[buf]);
		}
		seg = seg_end;
	}
}

// the mbarriers of one CTA: STAGES stage pairs and kRedBufs exchange pairs
template <int STAGES>
__device__ __forceinline__ Bars init_bars(uint64_t *base)
{
	Bars b{base, base + STAGES, base + 2 * STAGES, base + 2 * STAGES + kRedBufs};
	if (threadIdx.x < STAGES) {
		mbar_init(&b.full[threadIdx.x], 1);
		mbar_init(&b.empty[threadIdx.x], kMmaWarps);
	}
	if (threadIdx.x < kRedBufs) {
		mbar_init(&b.rfull[threadIdx.x], kMmaWarps);
		mbar_init(&b.rempty[threadIdx.x], 1);
	}
	return b;
}

// Stage shape of a matrix pass: WB blocks per math warp, MT m-tiles per
// item.  2048-column stages when cols is a multiple of 2048; a single
// 1024-column matrix takes two m-tiles per item (32 rows, four K slices)
// so that a stage still holds 16 slots of weights; else cols/256 blocks
// per warp for 256/512/1024 columns.  {0, 0}: not supported.
struct Shape {
	int wb, mt;
};

__host__ __device__ inline Shape pick_shape(int cols, bool dual)
{
	if (cols % 2048 == 0)
		return {8, 1};
	if (cols == 1024 && !dual)
		return {8, 2};
	if (cols == 1024 || cols == 512 || cols == 256)
		return {cols / 256, 1};
	return {0, 0};
}

}  // namespace moe
