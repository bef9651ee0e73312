// expert_gemm.cu — prefill-sized grouped expert GEMM on the 5th-generation
// tensor cores (tcgen05, accumulators in tensor memory).
//
// For every active expert e:
//   gate/up: H = silu(X_e W_gate^T) * (X_e W_up^T)     (DUAL)
//   down:    Y = H_e W_down^T                          (single)
// Activations are fp16 hi/lo rows in pair order (X_e, H_e contiguous per
// expert), natural column order.  Weights stay Q8_0/Q4_0 GGUF blocks in HBM.
//
// Work item = (active expert, weight row block, 128 pairs).  The MMA is
// D[pair][row] = A[pair][k] . B[row][k] with M = 128 pairs and N = 256
// weight rows: gate rows [128 rb, +128) stacked on the same up rows (DUAL),
// or rows [256 rb, +256) (single).  Each activation tile is read once per
// 256 weight rows, which keeps the operand reads from shared memory under
// its bandwidth.  One CTA per SM walks the items b, b + grid, ... with
// warp-specialised roles:
//   warp 0   lane 0: per 32-column slice (one block), TMA copies of a raw
//            window of the two weight halves (128 rows x 48 bytes Q8_0 / 32
//            bytes Q4_0: the slice's block starting on the 16-byte boundary
//            below it; one tensor map per expert matrix, built when the
//            layer is created)
//            lane 1: TMA tiles of the activations (128 rows x 32 columns, hi
//            and lo, 64-byte swizzle; rows past the end read as zeros)
//   warp 1   lane 0: issues tcgen05.mma (M 128, N 256, K 16, fp16 x fp16 ->
//            fp32) and commits to the slot and accumulator mbarriers
//   warps 2, 3, 8-13: dequantize each slice into w_hi = fp16(d * q) and
//            w_lo = fp16(d * q - w_hi) tiles (256 rows, K-major, 64-byte
//            swizzle)
//   warps 4-7: epilogue, one TMEM lane quadrant (32 pairs) each: tcgen05.ld,
//            SwiGLU (gate/up, stored as fp16 hi/lo) or nothing (down),
//            16-byte row-segment stores
// Tensor memory: two accumulator sets of 256 columns, so the epilogue of
// one item overlaps the MMAs of the next.  Shared memory holds 3
// activation slots, 8 weight slots (4 slices of hi/lo, so the dequant warps
// run ahead of the MMAs) and the raw ring; its bandwidth, shared by the MMA
// operand reads, the dequant stores and the TMA writes, is what bounds the
// kernel.
//
// Precision: each product is x_hi w_hi + x_lo w_hi + x_hi w_lo (three MMAs,
// the lo x lo term is below fp32 rounding), so weights and activations both
// carry about 22 significant bits; what remains is the tensor cores' fp32
// accumulation (about 2e-5 relative).  One fp16 term per operand is not
// enough for the north-star bar: at Mixtral-sized outputs (|y| ~ 10) its
// max-abs error reaches 5e-3 against the 2e-3 bound.
//
// Every wait is bounded (2 s of %globaltimer); an expired wait records an
// error code and the role keeps walking its loops without waiting, so the
// kernel ends.  Before the CTA ends, the copy issuers wait (bounded) for
// their last copies and the MMA issuer for its last MMAs; tensor memory is
// released in every case.
#include "expert_core.cuh"
#include "kernels.h"

#include <cuda.h>

namespace moe {

namespace {

constexpr int kGP = 128;             // pairs per item (MMA M)
constexpr int kGR = 256;             // weight rows per item (MMA N): two halves of 128
constexpr int kGH = 128;             // rows per half
constexpr int kGKS = 32;             // columns per slice (one block; a 64-byte swizzle row)
constexpr int kGThreads = 14 * 32;
constexpr int kProdWarp = 0, kMmaWarp = 1;
constexpr int kEpiFirst = 4;         // warps 4-7 (TMEM lane quadrants 0-3)
constexpr int kConvWarps = 8;        // warps 2, 3, 8-13: two per SM sub-partition
constexpr int kSmemMax = 232448;     // opt-in shared memory per block
constexpr int kStaticSmem = 3 * kMaxActive * 4 + 32;

__device__ __forceinline__ bool is_conv_warp(int w) { return w == 2 || w == 3 || w >= 8; }
__device__ __forceinline__ int conv_index(int w) { return w < 8 ? w - 2 : w - 6; }

template <int QT>
struct GemmLayout {
	static constexpr int BB = QT == kQ8_0 ? Q8_0_BYTES : Q4_0_BYTES;
	// a slice's block starts (34 s or 18 s bytes into the row) at most 14
	// bytes past a 16-byte boundary: the window covers it from there
	static constexpr int WIN = QT == kQ8_0 ? 48 : 32;
	static constexpr int RAW_UNIT = 2 * kGH * WIN;             // both halves: 12 / 8 KB
	static constexpr int ACT_HALF = kGP * kGKS * 2;            // 8 KB
	static constexpr int ACT_UNIT = 2 * ACT_HALF;              // x_hi + x_lo
	static constexpr int W_UNIT = kGR * kGKS * 2;              // 16 KB: 256 rows (hi or lo)
	static constexpr int ACT_SLOTS = 3, W_SLOTS = 8;
	// 1024-byte aligned regions: activation slots, weight slots, raw slots
	static constexpr int OFF_ACT = 0;
	static constexpr int OFF_W = OFF_ACT + ACT_SLOTS * ACT_UNIT;
	static constexpr int OFF_RAW = OFF_W + W_SLOTS * W_UNIT;
	static constexpr int NBARS_MAX = 48;
	static constexpr int AVAIL = kSmemMax - kStaticSmem - 1024 - NBARS_MAX * 8 - 16 - OFF_RAW;
	static constexpr int RAW_SLOTS = AVAIL / RAW_UNIT > 8 ? 8 : AVAIL / RAW_UNIT;
	static constexpr int OFF_BAR = OFF_RAW + RAW_SLOTS * RAW_UNIT;
	static constexpr int NBARS = 2 * RAW_SLOTS + 2 * ACT_SLOTS + 2 * W_SLOTS + 2 * 2 + 1;
	static constexpr int OFF_TMEM = OFF_BAR + NBARS * 8;
	static constexpr int BYTES = OFF_TMEM + 16;
	static constexpr int SMEM = BYTES + 1024;                 // room to align the base
	static_assert(RAW_SLOTS >= 3, "raw ring too small");
	static_assert(NBARS <= NBARS_MAX, "barrier area");
	static_assert(SMEM + kStaticSmem <= kSmemMax, "shared memory");
	static_assert(RAW_UNIT % 1024 == 0 && OFF_RAW % 1024 == 0, "slot alignment");
};

__device__ __forceinline__ uint64_t sw64_desc(uint32_t saddr)
{
	// K-major, 64-byte swizzle: start >> 4, LBO 16 B, SBO 512 B (8 rows of
	// 64 B), descriptor version 1, layout type 4
	return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) |
	       ((uint64_t)(512 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)4 << 61);
}

// fp16 x fp16 -> fp32, K-major A and B, M 128 (pairs), N 256 (weight rows)
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kGR >> 3) << 17) | ((uint32_t)(kGP >> 4) << 24);

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t acc)
{
	asm volatile(
		"{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
		"tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
		"l"(da), "l"(db), "r"(kIdesc), "r"(acc)
		: "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar)
{
	asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
			     smem_addr(bar))
		     : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory; map is a kernel parameter or a tensor
// map in global memory
__device__ __forceinline__ void tma_load_2d(void *dst, const void *map, int x, int y, uint64_t *bar)
{
	asm volatile(
		"cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
			smem_addr(dst)),
		"l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
		: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t addr, float (&v)[16])
{
	uint32_t r[16];
	asm volatile(
		"tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
		: "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
		  "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
		  "=r"(r[14]), "=r"(r[15])
		: "r"(addr));
	asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
	for (int j = 0; j < 16; j++)
		v[j] = __uint_as_float(r[j]);
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// the items of this CTA: (active expert a, row block rb, pair tile nt) in
// order a, rb, nt; item i of the whole list is handled by CTA i % grid.
// cum[a] = items of the active experts before a (cum[n_active] = all).
struct ItemWalk {
	const int32_t *en;   // [n_active] expert | pairs << 8
	const int32_t *cum;
	int n_active, rblocks;
	int a = 0, rb = 0, nt = 0, idx = 0;
	__device__ int tiles_of(int i) const
	{
		const int n = en[i] >> 8;
		return n / kGP + (n % kGP != 0);
	}
	__device__ bool done() const { return a >= n_active; }
	__device__ void seek()
	{
		while (a < n_active && cum[a + 1] <= idx)
			a++;
		if (a < n_active) {
			const int nts = tiles_of(a), rem = idx - cum[a];
			rb = rem / nts;
			nt = rem - rb * nts;
		}
	}
	__device__ void first()
	{
		a = 0;
		idx = blockIdx.x;
		seek();
	}
	__device__ void step()
	{
		idx += gridDim.x;
		seek();
	}
};

// two int8 codes (low byte first) -> half2 of the exact integers
__device__ __forceinline__ __half2 codes_to_h2(uint32_t w)
{
	const uint32_t biased = __byte_perm(w ^ 0x8080u, 0x64646464u, 0x4140);  // 1024 + q + 128
	return __hsub2(*reinterpret_cast<const __half2 *>(&biased),
		       __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));
}

// nibbles (bits 0-3 and 16-19 of w) -> half2 of (nib - 8)
__device__ __forceinline__ __half2 nibs_to_h2(uint32_t w)
{
	const uint32_t biased = (w & 0x000F000Fu) | 0x64006400u;  // 1024 + nib
	return __hsub2(*reinterpret_cast<const __half2 *>(&biased),
		       __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408)));
}

// Dequantize slice s (32 columns = one block) of both halves from a raw slot
// (half m, row r at m * 128 * WIN + r * WIN, the block from byte pad) into
// the hi and lo weight tiles: 256 rows x 32 columns fp16, K-major, 64-byte
// swizzle, half m at +8 KB * m.  hi = fp16(d q), lo = fp16(d q - hi)
// (exact: d q has at most 18 significant bits).  Unit (row r, 16-byte chunk
// c) = columns 8c..8c+7, stored at r * 64 + ((c ^ ((r >> 1) & 3)) * 16).
// Thread t owns chunk c = t % 4 of rows t / 4 + 64 k (k < 4), so every
// address is a fixed stride from its first; all loads are issued before the
// conversions.
template <int QT>
__device__ __forceinline__ void convert_slice(const uint8_t *raw, int pad, uint8_t *hi, uint8_t *lo,
					      int t)
{
	using GL = GemmLayout<QT>;
	constexpr int CH = kGKS / 8;                      // 16-byte chunks per row
	constexpr int U = kGR * CH / (kConvWarps * 32);
	constexpr int RSTEP = kConvWarps * 32 / CH;       // rows between a thread's units
	static_assert(RSTEP % 8 == 0, "swizzle phase must repeat");
	const int r0 = t / CH, c = t % CH;
	const uint8_t *b0 = raw + r0 * GL::WIN + pad;
	const int coff = QT == kQ8_0 ? 2 + 8 * c : 2 + 8 * (c & 1);
	const int o0 = r0 * 64 + ((c ^ ((r0 >> 1) & 3)) << 4);  // same phase for every unit
	uint32_t dq[U], w0[U], w1[U];
	// the 8 code bytes (at pad + 2 + 8c into the row, rows 16-byte aligned)
	// are 4-byte aligned when pad = 2 mod 4; otherwise (the same for every
	// thread of the slice) three aligned words are read and shifted by 16 bits
	if (pad & 2) {
#pragma unroll
		for (int k = 0; k < U; k++) {
			const uint8_t *b = b0 + k * RSTEP * GL::WIN;
			dq[k] = *reinterpret_cast<const uint16_t *>(b);
			const uint32_t *p = reinterpret_cast<const uint32_t *>(b + coff);
			w0[k] = p[0];
			w1[k] = p[1];
		}
	} else {
#pragma unroll
		for (int k = 0; k < U; k++) {
			const uint8_t *b = b0 + k * RSTEP * GL::WIN;
			dq[k] = *reinterpret_cast<const uint16_t *>(b);
			const uint32_t *p = reinterpret_cast<const uint32_t *>(b + coff - 2);
			const uint32_t a0 = p[0], a1 = p[1], a2 = p[2];
			w0[k] = __funnelshift_r(a0, a1, 16);
			w1[k] = __funnelshift_r(a1, a2, 16);
		}
	}
	const int sh = (QT == kQ4_0 && (c & 2)) ? 4 : 0;
#pragma unroll
	for (int k = 0; k < U; k++) {
		const __half d = __ushort_as_half((unsigned short)dq[k]);
		const __half2 d2 = __halves2half2(d, d);
		__half2 h[4];
		if (QT == kQ8_0) {
			h[0] = codes_to_h2(w0[k]);
			h[1] = codes_to_h2(w0[k] >> 16);
			h[2] = codes_to_h2(w1[k]);
			h[3] = codes_to_h2(w1[k] >> 16);
		} else {
			// elements 8c .. 8c+7: low nibbles of bytes 8(c&1).. for c < 2,
			// high nibbles of bytes 8(c&1).. for c >= 2
			const uint32_t x0 = w0[k] >> sh, x1 = w1[k] >> sh;
			// bytes b0 b1 b2 b3 of x0: elements 0..3; pairs (b0,b1), (b2,b3)
			h[0] = nibs_to_h2(__byte_perm(x0, 0, 0x5140));   // b0 -> bits 0-7, b1 -> 16-23
			h[1] = nibs_to_h2(__byte_perm(x0, 0, 0x5342));
			h[2] = nibs_to_h2(__byte_perm(x1, 0, 0x5140));
			h[3] = nibs_to_h2(__byte_perm(x1, 0, 0x5342));
		}
		uint4 oh, ol;
		__half2 *ph = reinterpret_cast<__half2 *>(&oh), *pl = reinterpret_cast<__half2 *>(&ol);
#pragma unroll
		for (int j = 0; j < 4; j++) {
			ph[j] = __hmul2(h[j], d2);                   // fp16(d * q), rounded once
			pl[j] = __hfma2(h[j], d2, __hneg2(ph[j]));   // d * q - hi, exact
		}
		const int o = o0 + k * RSTEP * 64;               // rows 128.. continue at +8 KB
		*reinterpret_cast<uint4 *>(hi + o) = oh;
		*reinterpret_cast<uint4 *>(lo + o) = ol;
	}
}

template <int QT, bool DUAL>
__global__ void __launch_bounds__(kGThreads, 1)
expert_gemm_kernel(GemmArgs a, const __grid_constant__ CUtensorMap xmap)
{
	using GL = GemmLayout<QT>;
	constexpr int RS = GL::RAW_SLOTS, XS = GL::ACT_SLOTS, WS = GL::W_SLOTS;
	extern __shared__ uint8_t smem_raw[];
	uint8_t *smem = reinterpret_cast<uint8_t *>(
		(reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
	uint64_t *bars = reinterpret_cast<uint64_t *>(smem + GL::OFF_BAR);
	uint64_t *raw_full = bars, *raw_empty = raw_full + RS;
	uint64_t *x_full = raw_empty + RS, *x_empty = x_full + XS;
	uint64_t *w_full = x_empty + XS, *w_empty = w_full + WS;
	uint64_t *acc_full = w_empty + WS, *acc_empty = acc_full + 2, *drain = acc_empty + 2;
	uint32_t *tslot = reinterpret_cast<uint32_t *>(smem + GL::OFF_TMEM);
	// routing tables
	__shared__ int32_t en_s[kMaxActive], off_s[kMaxActive], cum_s[kMaxActive + 1];
	__shared__ int n_active_s;

	const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
	if (tid == 0) {
		n_active_s = *a.n_active;
		for (int i = 0; i < RS; i++) {
			mbar_init(&raw_full[i], 1);
			mbar_init(&raw_empty[i], kConvWarps);
		}
		for (int i = 0; i < XS; i++) {
			mbar_init(&x_full[i], 1);
			mbar_init(&x_empty[i], 1);
		}
		for (int i = 0; i < WS; i++) {
			mbar_init(&w_full[i], kConvWarps);
			mbar_init(&w_empty[i], 1);
		}
		for (int i = 0; i < 2; i++) {
			mbar_init(&acc_full[i], 1);
			mbar_init(&acc_empty[i], 4);
		}
		mbar_init(drain, 1);
		fence_mbar_init();
	}
	if (warp == kMmaWarp) {
		asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
				     smem_addr(tslot)),
			     "r"(512));
		asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
	}
	__syncthreads();
	const int rows = a.rows, cols = a.cols;
	const int nslice = cols / kGKS;
	// DUAL: 128 gate rows + the same up rows; single: 256 rows (a last
	// block of 128: the weight map reads zeros past the matrix and the
	// epilogue stores only the rows that exist)
	const int rblocks = DUAL ? rows / kGH : (rows + kGR - 1) / kGR;
	if (warp == 0) {
		// routing tables and the item prefix (32 experts per shuffle scan)
		int acc = 0;
		for (int base = 0; base < n_active_s; base += 32) {
			const int i = base + lane;
			int items = 0;
			if (i < n_active_s) {
				const int e = a.active[i], n = a.counts[e];
				en_s[i] = e | (n << 8);
				off_s[i] = a.offsets[e];
				items = rblocks * (n / kGP + (n % kGP != 0));
			}
			int incl = items;
#pragma unroll
			for (int o = 1; o < 32; o <<= 1) {
				const int v = __shfl_up_sync(0xffffffffu, incl, o);
				if (lane >= o)
					incl += v;
			}
			if (i < n_active_s)
				cum_s[i] = acc + incl - items;
			acc += __shfl_sync(0xffffffffu, incl, 31);
		}
		if (lane == 0)
			cum_s[n_active_s] = acc;
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = *tslot;
	ItemWalk w{en_s, cum_s, n_active_s, rblocks};
	bool failed = false;
	auto wait = [&](uint64_t *bar, uint32_t parity) {
		if (!failed && !mbar_wait(bar, parity)) {
			failed = true;
			atomicExch(a.err, 2);
		}
	};
	const CUtensorMap *maps1 = static_cast<const CUtensorMap *>(a.maps1);
	const CUtensorMap *maps2 = static_cast<const CUtensorMap *>(a.maps2);

	if (warp == kProdWarp && lane == 0) {
		// ---- raw windows of both halves, one slot per slice
		uint32_t j = 0, n_issued = 0;
		for (w.first(); !w.done(); w.step()) {
			const int e = en_s[w.a] & 255;
			for (int s = 0; s < nslice; s++, j++) {
				const int st = j % RS;
				if (j >= RS)
					wait(&raw_empty[st], ((j / RS) - 1) & 1);
				if (failed)
					continue;
				const int x = ((s * GL::BB) & ~15) / 2;   // 16-bit words
				uint8_t *dst = smem + GL::OFF_RAW + st * GL::RAW_UNIT;
				mbar_arrive_expect_tx(&raw_full[st], (uint32_t)GL::RAW_UNIT);
				if (DUAL) {
					tma_load_2d(dst, &maps1[e], x, w.rb * kGH, &raw_full[st]);
					tma_load_2d(dst + kGH * GL::WIN, &maps2[e], x, w.rb * kGH, &raw_full[st]);
				} else {
					tma_load_2d(dst, &maps1[e], x, w.rb * kGR, &raw_full[st]);
					tma_load_2d(dst + kGH * GL::WIN, &maps1[e], x, w.rb * kGR + kGH, &raw_full[st]);
				}
				n_issued++;
			}
		}
		// no copy may still be landing when the CTA ends (after an error too)
		for (uint32_t k = n_issued > (uint32_t)RS ? n_issued - RS : 0; k < n_issued; k++)
			mbar_wait(&raw_full[k % RS], (k / RS) & 1);
	} else if (warp == kProdWarp && lane == 1) {
		// ---- activation tiles (hi at column 64 s, lo at cols + 64 s)
		uint32_t i = 0, n_issued = 0;
		for (w.first(); !w.done(); w.step()) {
			const int row0 = off_s[w.a] + w.nt * kGP;
			for (int s = 0; s < nslice; s++, i++) {
				const int st = i % XS;
				if (i >= XS)
					wait(&x_empty[st], ((i / XS) - 1) & 1);
				if (failed)
					continue;
				uint8_t *dst = smem + GL::OFF_ACT + st * GL::ACT_UNIT;
				mbar_arrive_expect_tx(&x_full[st], GL::ACT_UNIT);
				tma_load_2d(dst, &xmap, s * kGKS, row0, &x_full[st]);
				tma_load_2d(dst + GL::ACT_HALF, &xmap, cols + s * kGKS, row0, &x_full[st]);
				n_issued++;
			}
		}
		for (uint32_t k = n_issued > (uint32_t)XS ? n_issued - XS : 0; k < n_issued; k++)
			mbar_wait(&x_full[k % XS], (k / XS) & 1);
	} else if (is_conv_warp(warp)) {
		// ---- dequantize each slice into a hi/lo pair of weight slots
		const int ct = conv_index(warp) * 32 + lane;
		uint32_t i = 0, j = 0;
		for (w.first(); !w.done(); w.step()) {
			for (int s = 0; s < nslice; s++, j++, i += 2) {
				const int rs = j % RS, sh = i % WS, sl = (i + 1) % WS;
				wait(&raw_full[rs], (j / RS) & 1);
				if (i >= WS)
					wait(&w_empty[sh], ((i / WS) - 1) & 1);
				if (i + 1 >= WS)
					wait(&w_empty[sl], (((i + 1) / WS) - 1) & 1);
				if (!failed)
					convert_slice<QT>(smem + GL::OFF_RAW + rs * GL::RAW_UNIT, (s * GL::BB) & 15,
							  smem + GL::OFF_W + sh * GL::W_UNIT,
							  smem + GL::OFF_W + sl * GL::W_UNIT, ct);
				fence_proxy_async();   // generic writes -> tensor-core reads
				__syncwarp();
				if (lane == 0) {
					mbar_arrive(&w_full[sh]);
					mbar_arrive(&w_full[sl]);
					mbar_arrive(&raw_empty[rs]);
				}
			}
		}
	} else if (warp == kMmaWarp && lane == 0) {
		// ---- tensor-core issue: x_hi w_hi + x_lo w_hi, then x_hi w_lo
		uint32_t i = 0, xi = 0, it = 0;
		for (w.first(); !w.done(); w.step(), it++) {
			const int ab = it & 1;
			if (it >= 2)
				wait(&acc_empty[ab], ((it >> 1) - 1) & 1);
			tc_fence_after();
			const uint32_t d = tmem + ab * 256;
			for (int s = 0; s < nslice; s++, xi++, i += 2) {
				const int xs = xi % XS, wh = i % WS, wl = (i + 1) % WS;
				wait(&x_full[xs], (xi / XS) & 1);
				const uint32_t sx = smem_addr(smem + GL::OFF_ACT + xs * GL::ACT_UNIT);
				wait(&w_full[wh], (i / WS) & 1);
				tc_fence_after();
				if (!failed) {
					const uint32_t sw = smem_addr(smem + GL::OFF_W + wh * GL::W_UNIT);
#pragma unroll
					for (int k = 0; k < kGKS / 16; k++) {
						umma(d, sw64_desc(sx + k * 32), sw64_desc(sw + k * 32),
						     (s > 0 || k > 0) ? 1u : 0u);
						umma(d, sw64_desc(sx + GL::ACT_HALF + k * 32), sw64_desc(sw + k * 32), 1u);
					}
				}
				umma_commit(&w_empty[wh]);
				wait(&w_full[wl], ((i + 1) / WS) & 1);
				tc_fence_after();
				if (!failed) {
					const uint32_t sw = smem_addr(smem + GL::OFF_W + wl * GL::W_UNIT);
#pragma unroll
					for (int k = 0; k < kGKS / 16; k++)
						umma(d, sw64_desc(sx + k * 32), sw64_desc(sw + k * 32), 1u);
				}
				umma_commit(&w_empty[wl]);
				umma_commit(&x_empty[xs]);
			}
			umma_commit(&acc_full[ab]);
		}
		// every MMA has completed before tensor memory is released
		umma_commit(drain);
		mbar_wait(drain, 0);
	} else if (warp >= kEpiFirst && warp < kEpiFirst + 4) {
		// ---- epilogue: TMEM lane quadrant q = pairs 32q .. 32q + 31 of the item
		const int q = warp - kEpiFirst;
		uint32_t it = 0;
		for (w.first(); !w.done(); w.step(), it++) {
			const int ab = it & 1;
			wait(&acc_full[ab], (it >> 1) & 1);
			tc_fence_after();
			const int n = 32 * q + lane;                          // this thread's pair
			const bool valid = n < (en_s[w.a] >> 8) - w.nt * kGP;
			const int pos = off_s[w.a] + w.nt * kGP + n;
			const uint32_t tq = tmem + ab * 256 + ((uint32_t)(32 * q) << 16);
			if (DUAL) {
				__half *oh = a.out16 + (int64_t)pos * 2 * rows + w.rb * kGH;
				for (int c0 = 0; c0 < kGH; c0 += 16) {
					float g[16], u[16];
					tmem_ld16(tq + c0, g);
					tmem_ld16(tq + kGH + c0, u);
					if (failed || !valid)
						continue;
					uint4 vh[2], vl[2];
					__half *ph = reinterpret_cast<__half *>(vh), *pl = reinterpret_cast<__half *>(vl);
#pragma unroll
					for (int j = 0; j < 16; j++) {
						const float h = swiglu(g[j], u[j]);
						ph[j] = __float2half_rn(h);
						pl[j] = __float2half_rn(h - __half2float(ph[j]));
					}
					uint4 *dh = reinterpret_cast<uint4 *>(oh + c0), *dl = reinterpret_cast<uint4 *>(oh + rows + c0);
					dh[0] = vh[0];
					dh[1] = vh[1];
					dl[0] = vl[0];
					dl[1] = vl[1];
				}
			} else {
				const int orow = valid ? (a.out_perm ? a.perm[pos] : pos) : 0;
				float *o = a.out + (int64_t)orow * rows + w.rb * kGR;
				const int ncols = min(kGR, rows - w.rb * kGR);  // warp-uniform
				for (int c0 = 0; c0 < ncols; c0 += 16) {
					float y[16];
					tmem_ld16(tq + c0, y);
					if (failed || !valid)
						continue;
					float4 *dst = reinterpret_cast<float4 *>(o + c0);
#pragma unroll
					for (int j = 0; j < 4; j++)
						dst[j] = make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
				}
			}
			tc_fence_before();
			__syncwarp();
			if (lane == 0)
				mbar_arrive(&acc_empty[ab]);
		}
	}
	tc_fence_before();
	__syncthreads();
	if (warp == kMmaWarp) {
		tc_fence_after();
		asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
	}
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
				  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
				  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
				  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
	static EncodeTiledFn fn = nullptr;
	if (!fn) {
		cudaDriverEntryPointQueryResult q;
		void *p = nullptr;
		if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
			    cudaSuccess &&
		    q == cudaDriverEntryPointSuccess)
			fn = reinterpret_cast<EncodeTiledFn>(p);
	}
	return fn;
}

template <int QT, bool DUAL>
cudaError_t launch_gemm_t(const GemmArgs &a, int64_t in_rows, cudaStream_t st)
{
	using GL = GemmLayout<QT>;
	// activations: [in_rows][2][cols] fp16 (hi, lo), tile 32 columns x 128
	// rows, 64-byte swizzle
	CUtensorMap map;
	EncodeTiledFn enc = encode_fn();
	if (!enc)
		return cudaErrorNotSupported;
	const cuuint64_t dims[2] = {(cuuint64_t)(2 * a.cols), (cuuint64_t)in_rows};
	const cuuint64_t strides[1] = {(cuuint64_t)a.cols * 4};
	const cuuint32_t box[2] = {(cuuint32_t)kGKS, (cuuint32_t)kGP}, es[2] = {1, 1};
	if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(a.in16), dims, strides,
		box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
		CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
		return cudaErrorInvalidValue;
	auto fn = expert_gemm_kernel<QT, DUAL>;
	cudaError_t e = ensure_smem(fn, GL::SMEM);
	if (e != cudaSuccess)
		return e;
	fn<<<sm_count(), kGThreads, GL::SMEM, st>>>(a, map);
	return cudaGetLastError();
}

}  // namespace

bool expert_gemm_supported(int qtype, int rows, int cols, int dual)
{
	// cols % 256: rows of 16-byte multiples for the weight tensor maps;
	// rows % 128 (single: a last item of 128 rows is masked)
	return (qtype == kQ8_0 || qtype == kQ4_0) && rows % kGH == 0 && cols % 256 == 0 &&
	       encode_fn() != nullptr;
}

bool encode_weight_map(void *map, const void *w, int qtype, int rows, int cols)
{
	// a weight matrix as [rows][row_bytes / 2] 16-bit words; box = one raw
	// window (128 rows x WIN bytes), no swizzle; windows reaching past the
	// row end read zeros
	EncodeTiledFn enc = encode_fn();
	if (!enc || !w || (uintptr_t)w % 16)
		return false;
	const int bb = qtype == kQ8_0 ? Q8_0_BYTES : Q4_0_BYTES;
	const int64_t row_bytes = (int64_t)(cols / QK) * bb;
	const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 2), (cuuint64_t)rows};
	const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
	const int win = qtype == kQ8_0 ? GemmLayout<kQ8_0>::WIN : GemmLayout<kQ4_0>::WIN;
	const cuuint32_t box[2] = {(cuuint32_t)(win / 2), (cuuint32_t)kGH}, es[2] = {1, 1};
	return enc(static_cast<CUtensorMap *>(map), CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(w),
		   dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
		   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t weight_map_bytes() { return sizeof(CUtensorMap); }

cudaError_t launch_expert_gemm(const GemmArgs &a, int64_t in_rows, cudaStream_t st)
{
	if (a.n_local <= 0 || in_rows <= 0)
		return cudaSuccess;
	if (!expert_gemm_supported(a.qtype, a.rows, a.cols, a.dual) || !a.maps1 ||
	    (a.dual && !a.maps2) || (uintptr_t)a.in16 % 16)
		return cudaErrorInvalidValue;
	if (a.qtype == kQ8_0)
		return a.dual ? launch_gemm_t<kQ8_0, true>(a, in_rows, st)
			      : launch_gemm_t<kQ8_0, false>(a, in_rows, st);
	return a.dual ? launch_gemm_t<kQ4_0, true>(a, in_rows, st)
		      : launch_gemm_t<kQ4_0, false>(a, in_rows, st);
}

// out[pos][0][k] = fp16(x[t][k]), out[pos][1][k] = fp16(x[t][k] - hi) with
// t = perm[pos] / K: the tokens in pair order, hi/lo
__global__ void gather_split_kernel(const float *__restrict__ x, const int32_t *__restrict__ perm,
				    int64_t pairs, int cols, int K, __half *__restrict__ out)
{
	const int c4 = cols / 4;
	const int64_t total = pairs * c4;
	for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
	     i += (int64_t)gridDim.x * blockDim.x) {
		const int64_t pos = i / c4;
		const int k = (int)(i - pos * c4);
		const int64_t src = perm ? perm[pos] / K : pos;  // no perm: rows in order (dense GEMM)
		const float4 v = reinterpret_cast<const float4 *>(x + src * cols)[k];
		const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
		const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
		__half2 hi[2] = {h0, h1};
		__half2 lo[2] = {__floats2half2_rn(v.x - f0.x, v.y - f0.y),
				 __floats2half2_rn(v.z - f1.x, v.w - f1.y)};
		__half *row = out + pos * 2 * cols;
		reinterpret_cast<uint2 *>(row)[k] = *reinterpret_cast<uint2 *>(hi);
		reinterpret_cast<uint2 *>(row + cols)[k] = *reinterpret_cast<uint2 *>(lo);
	}
}

cudaError_t launch_gather_split(const float *x, const int32_t *perm, int64_t pairs, int cols,
				int K, __half *out, cudaStream_t st)
{
	if (pairs == 0)
		return cudaSuccess;
	if (cols % 4 || (uintptr_t)x % 16 || (uintptr_t)out % 8)
		return cudaErrorInvalidValue;
	int64_t blocks = (pairs * cols / 4 + 255) / 256;
	if (blocks > (int64_t)sm_count() * 16)
		blocks = (int64_t)sm_count() * 16;
	gather_split_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, perm, pairs, cols, K, out);
	return cudaGetLastError();
}

}  // namespace moe
