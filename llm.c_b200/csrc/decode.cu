// decode.cu — the whole MoE layer of a decode-sized batch (T <= 64 tokens)
// in one persistent kernel: one CTA per SM, launched cooperatively so that
// all CTAs are resident and can meet at grid-wide barriers.
//
// It computes what models/olmoe/olmoe.c:343-407 (and llama.c:393-457 with
// renormalisation) compute, phase by phase:
//
//   P0  router logits (matmul.c:91-131 lane order, exact) by tiles of
//       8 or 16 tokens x 8 experts spread over the CTAs (up to 8 tokens: one
//       expert per CTA), each tile staged into shared memory by bulk
//       copies; every CTA also writes its share of the fp16 hi/lo split of
//       x that the expert phases read.
//   --  grid barrier
//   P1  CTA t computes softmax + top-k (nn.c:221-308) of token t; grid
//       barrier; then every CTA reads the selected (token, slot) pairs and
//       computes their stable dispatch by expert into its own shared
//       memory (redundant, but cheaper than another barrier); CTA 0 writes
//       the dispatch to global memory for the host.  Up to 11 tokens on one
//       rank, every CTA ranks every token itself (one thread per (token,
//       expert) up to 5 tokens) and no second barrier is needed; up to 32
//       pairs, one warp dispatches them.
//   P2  gate/up + SwiGLU over (active expert, 8-row) items — the expert
//       pipeline of expert_core.cuh, writing h as fp16 hi/lo rows.
//   --  grid barrier among the math and epilogue warps.  The producer warp
//       does not wait: down weights do not depend on h, so it keeps
//       streaming them into the stage ring while P2 drains elsewhere.
//   P3  down over (active expert, 16-row) items, writing one fp32 row per
//       (token, slot) pair.
//   --  grid barrier
//   P4  combine: out[t] = sum_s y[t,s] / (1/w[t,s]) in slot order
//       (olmoe.c:397-404); spread over every CTA, the divisions cost
//       little here, while in P3's epilogue they held back the down rows
//       the quotients in slot order, spread over every thread of the grid.
//
// Replacing five launches (and their drain / ramp-up) by one also keeps the
// routing tables in shared memory, where the expert phases read them.
//
// Every wait is bounded (mbarriers and the grid barrier: 2 s); an expired
// wait records an error code in a device flag that the host reads, and the
// kernel runs to its end without waiting further.
#include "expert_core.cuh"
#include "kernels.h"
#include "route_core.cuh"

namespace moe {

// per-warp scratch of the CTA-local top-k (P1, few tokens): logits [64],
// weights [32], ids [32]
constexpr int kLocalTopkBytes = (64 + 32 + 32) * 4;

// router tile of P0: RT tokens x RE experts, whole 2048-column row chunks
// staged by 16 bulk copies (one per row, issued by 16 lanes at once).
// Warps 0-3 compute: for 16 SIMD lanes, warp w owns lane quad w and its
// threads are (token, pair of experts); for 8 lanes, warp w owns lane quad
// w & 1 and four experts, one per thread.  Each thread keeps its lanes' fp32
// chains; the reference's halving tree over the lanes runs at the end, per
// logit, from shared memory.
template <int LANES>
struct RTile {
	static constexpr int LQ = LANES / 4;                 // lane quads per logit
	static constexpr int RT = 8;                         // tokens per tile
	static constexpr int RE = 8;                         // experts per tile
	static constexpr int EPT = LANES == 16 ? 2 : 1;      // experts per thread
	static constexpr int CH = 2048;                      // columns per chunk
	// 8 token rows of a warp read 8 distinct 16-byte bank groups
	static constexpr int RS = CH * 4 + 16;
	static constexpr int ROWS = RT + RE;
	static constexpr int PART = ROWS * RS;               // lane partials start here
	static constexpr int BYTES = PART + RT * RE * LANES * 4;
	static constexpr int NSLOT = 1;
};

// %globaltimer stamps per CTA (thread 0): phase ends and barrier exits
enum Stamp {
	kStStart, kStP0, kStB1, kStTopk, kStB1b, kStDispatch, kStP1, kStP2, kStB2, kStP3, kStB3,
	kStEnd, kStamps
};

struct DecodeSmem {
	// byte offsets after the stage ring
	static constexpr int EN = 0;                              // int32 [256]
	static constexpr int OFF = EN + kMaxActive * 4;            // int32 [256]
	static constexpr int PRE_GU = OFF + kMaxActive * 4;        // int32 [260]
	static constexpr int PRE_DN = PRE_GU + (kMaxActive + 4) * 4;
	static constexpr int WTS = PRE_DN + (kMaxActive + 4) * 4;  // f32   [1024] own pairs
	static constexpr int PERM = WTS + kDecodeMaxPairs * 4;     // int32 [2048] all pairs
	static constexpr int COUNTS = PERM + kDecodeMaxPairsAll * 4;  // int32 [256]
	static constexpr int OFFSETS = COUNTS + kMaxActive * 4;    // int32 [260]
	static constexpr int ACTIVE = OFFSETS + (kMaxActive + 4) * 4;  // int32 [256]
	static constexpr int NACT = ACTIVE + kMaxActive * 4;       // int32 [4]
	static constexpr int BARS = NACT + 16;                     // u64 bars
	static constexpr int END = BARS;                           // + bars
	// during P1 only: the dispatch scratch at the start of the stage ring,
	// the ids of the dispatched pairs behind it
	static constexpr int RING_IDS = 16 * 1024;
};
// u64 slots after the mbarriers: the router tile barrier, then the peer
// tables (row destinations of the replicated and the token-sharded
// exchange, this rank's gathered-token buffer in each rank)
constexpr int kPtrSlots = 1 + 3 * kMaxEpRanks;

template <int QT, int STAGES>
constexpr size_t decode_smem_bytes()
{
	return (size_t)STAGES * StageLayout<QT>::BYTES + StageLayout<QT>::RED +
	       StageLayout<QT>::EPI + DecodeSmem::END +
	       (2 * STAGES + 2 * kRedBufs + kPtrSlots) * 8;  // + router barrier, peer tables
}

// ---------------------------------------------------------------- grid barrier
__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long *p)
{
	unsigned long long v;
	asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
	return v;
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p)
{
	unsigned long long v;
	asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
	return v;
}

__device__ __forceinline__ void red_add_release_sys(unsigned long long *p, unsigned long long v)
{
	asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// cross-rank arrival wait: until *cnt reaches `want` (acquire, system
// scope), at most limit_ns; an expired wait records error 4
__device__ void wait_arrivals(const unsigned long long *cnt, unsigned long long want,
			      uint64_t limit_ns, int32_t *err)
{
	const uint64_t t0 = global_ns();
	while (ld_acquire_sys(cnt) < want) {
		if (global_ns() - t0 > limit_ns) {
			atomicExch(err, 4);
			return;
		}
		__nanosleep(64);
	}
}

// Grid barrier: bar[0] counts arrivals since the buffer was zeroed (a
// multiple of gridDim.x between barriers).  Each CTA's thread 0, after a
// CTA-level barrier, adds its arrival with release semantics (the CTA's
// writes before the barrier become visible with it) and polls the counter
// with acquire loads until the arrivals of this barrier are complete.  One
// hop instead of an arrival followed by a release of per-CTA flags: about
// 1-2 us per barrier on 148 CTAs instead of 3-5.  The poll is bounded.
constexpr int kGridFlagStride = 16;  // u64s: 128 bytes (the counter's line)

__device__ bool grid_sync(unsigned long long *bar, int32_t *err)
{
	const unsigned long long n = gridDim.x;
	unsigned long long ticket;
	asm volatile("atom.add.release.gpu.global.u64 %0, [%1], 1;" : "=l"(ticket) : "l"(bar) : "memory");
	const unsigned long long target = (ticket / n + 1) * n;
	if (ld_acquire_gpu(bar) < target) {
		const uint64_t t0 = global_ns();
		while (ld_acquire_gpu(bar) < target) {
			if (global_ns() - t0 > kWaitLimitNs) {
				atomicExch(err, 3);
				return false;
			}
			__nanosleep(20);
		}
	}
	return true;
}

size_t decode_barrier_bytes(int) { return kGridFlagStride * 8; }

__device__ __forceinline__ void bar_math_epi()
{
	// the math and epilogue warps (all warps but the producer)
	asm volatile("bar.sync 1, %0;" ::"n"(kCoreThreads - 32) : "memory");
}

__device__ __forceinline__ void stamp(uint64_t *stamps, int k)
{
	if (stamps && threadIdx.x == 0)
		stamps[blockIdx.x * kStamps + k] = global_ns();
}

// ---------------------------------------------------------------- P0 router
template <int LANES>
__device__ void router_tiles(const DecodeArgs &a, uint8_t *buf, uint64_t *rbar)
{
	using R = RTile<LANES>;
	const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
	const int n_tt = (a.T + R::RT - 1) / R::RT, n_et = a.NE / R::RE;
	const int nch = a.D / R::CH;
	// compute mapping (warps 0-3)
	const int lq = LANES == 16 ? warp : (warp & 1);
	const int tk = lane & 7;
	const int e_first = LANES == 16 ? 2 * (lane >> 3) : 4 * (warp >> 1) + (lane >> 3);
	float *part = reinterpret_cast<float *>(buf + R::PART);  // [RT][RE][LANES]
	uint32_t q = 0;  // chunks through the buffer (barrier phase)
	bool failed = false;
	for (int u = blockIdx.x; u < n_tt * n_et; u += gridDim.x) {
		const int t0 = (u / n_et) * R::RT, e0 = (u % n_et) * R::RE;
		const int nt = min(R::RT, a.T - t0);
		float acc[R::EPT][4];
#pragma unroll
		for (int k = 0; k < R::EPT; k++)
#pragma unroll
			for (int j = 0; j < 4; j++)
				acc[k][j] = 0.0f;
		for (int c = 0; c < nch; c++, q++) {
			if (warp == 0 && !failed) {
				// rows 0..RT-1: tokens (those past T are not copied); RT..: experts
				if (lane == 0)
					mbar_arrive_expect_tx(rbar, (uint32_t)((nt + R::RE) * R::CH * 4));
				__syncwarp();
				if (lane < R::ROWS && (lane >= R::RT || lane < nt)) {
					const float *src = lane < R::RT
								   ? a.x + (int64_t)(t0 + lane) * a.D
								   : a.router_w + (int64_t)(e0 + lane - R::RT) * a.D;
					fence_proxy_async();
					bulk_g2s(buf + lane * R::RS, src + (int64_t)c * R::CH, R::CH * 4, rbar);
				}
			}
			if (!failed && !mbar_wait(rbar, q & 1)) {
				failed = true;
				atomicExch(a.err, 2);
			}
			if (warp < 4 && !failed) {
				const float *xs = reinterpret_cast<const float *>(buf + tk * R::RS);
				const float *ws = reinterpret_cast<const float *>(buf + (R::RT + e_first) * R::RS);
#pragma unroll 4
				for (int st = 0; st < R::CH / LANES; st++) {
					const int col = st * LANES + lq * 4;
					const float4 xv = *reinterpret_cast<const float4 *>(xs + col);
#pragma unroll
					for (int k = 0; k < R::EPT; k++) {
						const float4 wv = *reinterpret_cast<const float4 *>(
							ws + k * (R::RS / 4) + col);
						acc[k][0] = __fmaf_rn(xv.x, wv.x, acc[k][0]);
						acc[k][1] = __fmaf_rn(xv.y, wv.y, acc[k][1]);
						acc[k][2] = __fmaf_rn(xv.z, wv.z, acc[k][2]);
						acc[k][3] = __fmaf_rn(xv.w, wv.w, acc[k][3]);
					}
				}
			}
			__syncthreads();  // the buffer is free again
		}
		// lane partials -> the reference's halving tree, one logit per thread
		if (warp < 4)
#pragma unroll
			for (int k = 0; k < R::EPT; k++)
#pragma unroll
				for (int j = 0; j < 4; j++)
					part[(tk * R::RE + e_first + k) * LANES + lq * 4 + j] = acc[k][j];
		__syncthreads();
		if (tid < R::RT * R::RE) {
			const int t = tid / R::RE, e = tid % R::RE;
			float l[LANES];
#pragma unroll
			for (int j = 0; j < LANES; j++)
				l[j] = part[tid * LANES + j];
#pragma unroll
			for (int h = LANES / 2; h >= 1; h /= 2)
#pragma unroll
				for (int j = 0; j < h; j++)
					l[j] = __fadd_rn(l[j], l[j + h]);
			if (t < nt)
				a.logits[(int64_t)(t0 + t) * a.NE + e0 + e] = __fadd_rn(0.0f, l[0]);
		}
		__syncthreads();
	}
}

// P0 for a few tokens (T <= 8): one expert per CTA (CTAs NE.. idle), so the
// router's latency is one 2048-column chunk of one row per CTA instead of
// eight.  The T token rows and the expert's row are staged by bulk copies;
// warp t computes token t: lane quad q (lane q < LANES / 4) carries the
// reference's SIMD lanes 4q..4q+3 (the same fp32 chains as router_tiles,
// matmul.c:91-105 with LANES lanes), and the halving tree over the lanes
// runs in lane 0 (the same additions in the same order).
constexpr int kSmallRouterT = 8;

template <int LANES>
__device__ void router_small(const DecodeArgs &a, uint8_t *buf, uint64_t *rbar)
{
	constexpr int CH = 2048, RS = CH * 4 + 16, LQ = LANES / 4;
	const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
	const int e = blockIdx.x;
	if (e >= a.NE)
		return;
	const int nch = a.D / CH;
	float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
	bool failed = false;
	for (int c = 0; c < nch; c++) {
		if (warp == 0) {
			// rows 0..T-1: tokens, row T: the expert
			if (lane == 0)
				mbar_arrive_expect_tx(rbar, (uint32_t)((a.T + 1) * CH * 4));
			__syncwarp();
			if (lane <= a.T) {
				const float *src = lane < a.T ? a.x + (int64_t)lane * a.D
							      : a.router_w + (int64_t)e * a.D;
				fence_proxy_async();
				bulk_g2s(buf + lane * RS, src + (int64_t)c * CH, CH * 4, rbar);
			}
		}
		if (!mbar_wait(rbar, c & 1)) {
			failed = true;
			atomicExch(a.err, 2);
		}
		if (!failed && warp < a.T && lane < LQ) {
			const float *xs = reinterpret_cast<const float *>(buf + warp * RS);
			const float *ws = reinterpret_cast<const float *>(buf + a.T * RS);
#pragma unroll 8
			for (int st = 0; st < CH / LANES; st++) {
				const int col = st * LANES + lane * 4;
				const float4 xv = *reinterpret_cast<const float4 *>(xs + col);
				const float4 wv = *reinterpret_cast<const float4 *>(ws + col);
				acc[0] = __fmaf_rn(xv.x, wv.x, acc[0]);
				acc[1] = __fmaf_rn(xv.y, wv.y, acc[1]);
				acc[2] = __fmaf_rn(xv.z, wv.z, acc[2]);
				acc[3] = __fmaf_rn(xv.w, wv.w, acc[3]);
			}
		}
		__syncthreads();  // the buffer is free again
		if (failed)
			break;
	}
	if (warp < a.T && !failed) {
		// lane j of the reference's LANES sits in lane j / 4, slot j % 4
		float l[LANES];
#pragma unroll
		for (int j = 0; j < LANES; j++)
			l[j] = __shfl_sync(0xffffffffu, acc[j % 4], j / 4);
		if (lane == 0) {
#pragma unroll
			for (int h = LANES / 2; h >= 1; h /= 2)
#pragma unroll
				for (int j = 0; j < h; j++)
					l[j] = __fadd_rn(l[j], l[j + h]);
			a.logits[(int64_t)warp * a.NE + e] = __fadd_rn(0.0f, l[0]);
		}
	}
}

// ---------------------------------------------------------------- the kernel
template <int QT, int LANES, int WB_GU, int WB_DN, int MT_DN, int STAGES>
__global__ void __launch_bounds__(kCoreThreads, 1) moe_decode_kernel(DecodeArgs a)
{
	extern __shared__ __align__(128) uint8_t smem[];
	using SL = StageLayout<QT>;
	using DS = DecodeSmem;
	uint8_t *tail = smem + STAGES * SL::BYTES;
	float4 *red = reinterpret_cast<float4 *>(tail);
	float *stg = reinterpret_cast<float *>(tail + SL::RED);
	uint8_t *tb = tail + SL::RED + SL::EPI;
	int32_t *en = reinterpret_cast<int32_t *>(tb + DS::EN);
	int32_t *off = reinterpret_cast<int32_t *>(tb + DS::OFF);
	int32_t *pre_gu = reinterpret_cast<int32_t *>(tb + DS::PRE_GU);
	int32_t *pre_dn = reinterpret_cast<int32_t *>(tb + DS::PRE_DN);
	float *wts_s = reinterpret_cast<float *>(tb + DS::WTS);
	int32_t *perm_s = reinterpret_cast<int32_t *>(tb + DS::PERM);
	int32_t *counts_s = reinterpret_cast<int32_t *>(tb + DS::COUNTS);
	int32_t *offsets_s = reinterpret_cast<int32_t *>(tb + DS::OFFSETS);
	int32_t *active_s = reinterpret_cast<int32_t *>(tb + DS::ACTIVE);
	int32_t *nact_s = reinterpret_cast<int32_t *>(tb + DS::NACT);
	uint64_t *bars = reinterpret_cast<uint64_t *>(tb + DS::BARS);
	uint64_t *rbar = bars + 2 * STAGES + 2 * kRedBufs;  // router tile buffer

	const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
	const int T = a.T, D = a.D, F = a.F, NE = a.NE, K = a.K;
	stamp(a.stamps, kStStart);
	const Bars b = init_bars<STAGES>(bars);
	if (tid == 0)
		mbar_init(rbar, 1);
	// expert parallelism: this launch's number (the same on every rank, as
	// every rank runs the same launches) and, by its parity, the half of
	// each exchange buffer it writes -- a rank one launch ahead writes the
	// other half, so it never overwrites rows that are still being combined
	const bool ep = a.world > 1;
	const bool shard = ep && a.shard;
	const unsigned long long epoch = ep ? *reinterpret_cast<volatile unsigned long long *>(a.launches) + 1 : 0;
	// the routing arrivals count token-sharded launches only
	const unsigned long long shard_epoch =
		shard ? *reinterpret_cast<volatile unsigned long long *>(a.shard_launches) + 1 : 0;
	const int64_t half_off = (int64_t)(epoch & 1) * a.ybuf_half;
	float *Y = ep ? a.ybuf[a.rank] + half_off : a.Y;
	// peer tables (smem): the other ranks' Y halves (replicated tokens),
	// every rank's Y half (token-sharded, indexed by rank), and this rank's
	// rows in every rank's gathered-token buffer (token-sharded)
	float **ypeers = reinterpret_cast<float **>(rbar + 1);
	float **yall = ypeers + kMaxEpRanks;
	__half **xgl = reinterpret_cast<__half **>(yall + kMaxEpRanks);
	if (ep && tid < a.world) {
		if (tid != a.rank)
			ypeers[tid - (tid > a.rank)] = a.ybuf[tid] + half_off;
		yall[tid] = a.ybuf[tid] + half_off;
		if (shard)
			xgl[tid] = a.xg[tid] + (int64_t)a.rank * T * 2 * D;
	}
	const uint64_t ep_wait = a.ep_wait_ns ? a.ep_wait_ns : kWaitLimitNs;
	fence_mbar_init();
	__syncthreads();

	// ------------------------------------------------ P0: logits + x split
	// The top-k of token t runs after barrier 1 on CTA (units + t) % grid,
	// normally a CTA without router work.  Such a CTA first runs the top-k
	// once on dummy logits, so that its code is in the SM's instruction cache
	// (it is otherwise fetched cold, from memory, when the result is needed).
	// a few tokens and enough CTAs: one expert per CTA (router_small)
	const bool small_router = T <= kSmallRouterT && NE <= (int)gridDim.x;
	const int units = small_router
				  ? NE
				  : ((T + RTile<LANES>::RT - 1) / RTile<LANES>::RT) * (NE / RTile<LANES>::RE);
	const int topk_first = units % (int)gridDim.x;  // CTA of token 0
	const int my_token0 = ((int)blockIdx.x - topk_first + (int)gridDim.x) % (int)gridDim.x;
	// few tokens on one rank: P1 ranks every token on every CTA (see there)
	const bool local_topk = !shard && T <= (int)(blockDim.x / 32) && NE <= 64;
	if (!local_topk && (int)blockIdx.x >= units && my_token0 < T && warp == 0) {
		float *lg = reinterpret_cast<float *>(smem);
		float *sel = lg + kMaxActive;
		int32_t *dummy = reinterpret_cast<int32_t *>(sel + 2 * K);
		for (int e = lane; e < NE; e += 32)
			lg[e] = 0.0f;
		__syncwarp();
		topk_token<LANES>(lg, nullptr, NE, K, a.mode_exact, a.renorm, sel,
				  reinterpret_cast<int32_t *>(sel + K), dummy, reinterpret_cast<float *>(dummy + K),
				  nullptr, nullptr);
	}
	if (small_router)
		router_small<LANES>(a, smem, rbar);
	else
		router_tiles<LANES>(a, smem, rbar);
	{
		// the fp16 hi/lo split of x that the expert phases read, 8 columns
		// per thread and 16-byte stores; token-sharded, into this rank's rows
		// of every rank's gathered-token buffer (over NVLink for the others)
		__half *xl = shard ? xgl[a.rank] : a.x16;
		const int64_t groups = (int64_t)T * D / 8;
		for (int64_t g = (int64_t)blockIdx.x * blockDim.x + tid; g < groups;
		     g += (int64_t)gridDim.x * blockDim.x) {
			const int64_t r = g * 8 / D;
			const int k = (int)(g * 8 - r * D);
			__align__(16) __half hi[8], lo[8];
#pragma unroll
			for (int j = 0; j < 8; j++) {
				const float v = __ldg(a.x + r * D + (QT == kQ4_0 ? q4_src(k + j) : k + j));
				hi[j] = __float2half_rn(v);
				lo[j] = __float2half_rn(__fsub_rn(v, __half2float(hi[j])));
			}
			const uint4 vh = *reinterpret_cast<const uint4 *>(hi);
			const uint4 vl = *reinterpret_cast<const uint4 *>(lo);
			*reinterpret_cast<uint4 *>(xl + r * 2 * D + k) = vh;
			*reinterpret_cast<uint4 *>(xl + r * 2 * D + D + k) = vl;
			if (shard)
				for (int q = 0; q < a.world; q++)
					if (q != a.rank) {
						__half *xp = xgl[q] + r * 2 * D + k;
						*reinterpret_cast<uint4 *>(xp) = vh;
						*reinterpret_cast<uint4 *>(xp + D) = vl;
					}
		}
	}
	__syncthreads();
	stamp(a.stamps, kStP0);
	if (tid == 0)
		grid_sync(a.gbar, a.err);
	__syncthreads();
	stamp(a.stamps, kStB1);

	// ------------------------------------------------ P1: routing
	// softmax + top-k of token t by warp 0 of CTA (units + t) % grid.  A few
	// tokens on one rank: every CTA ranks every token itself instead (warp t
	// takes token t), which saves the second grid barrier and a hop through
	// global memory; CTA 0 writes the routing for the host.
	int32_t *ids_all = reinterpret_cast<int32_t *>(smem + DS::RING_IDS);
	float *wtok = reinterpret_cast<float *>(smem + DS::RING_IDS + kDecodeMaxPairsAll * 4);
	{
		float *lg = reinterpret_cast<float *>(smem);                 // [NE]
		float *sel = lg + kMaxActive;                                // [2K]
		if (local_topk && T * 64 <= (int)blockDim.x) {
			// one thread per (token, expert)
			topk_tokens_cta<LANES>(a.logits, a.router_bias, T, NE, K, a.mode_exact, a.renorm,
					       reinterpret_cast<float *>(smem), ids_all, wtok,
					       blockIdx.x == 0 ? a.ids : nullptr,
					       blockIdx.x == 0 ? a.wts : nullptr);
		} else if (local_topk) {
			if (warp < T) {
				float *lgw = reinterpret_cast<float *>(smem + warp * kLocalTopkBytes);
				float *sw = lgw + 64;
				int32_t *sid = reinterpret_cast<int32_t *>(sw + 32);
				for (int e = lane; e < NE; e += 32)
					lgw[e] = __ldcg(a.logits + (int64_t)warp * NE + e);
				__syncwarp();
				topk_token<LANES>(lgw, a.router_bias, NE, K, a.mode_exact, a.renorm, sw, sid,
						  ids_all + warp * K, wtok + warp * K, nullptr, nullptr);
				if (blockIdx.x == 0)
					for (int q = lane; q < K; q += 32) {
						a.ids[(int64_t)warp * K + q] = ids_all[warp * K + q];
						a.wts[(int64_t)warp * K + q] = wtok[warp * K + q];
					}
			}
		}
		for (int t = my_token0; !local_topk && t < T; t += gridDim.x) {
			if (warp == 0) {
				for (int e = lane; e < NE; e += 32)
					lg[e] = __ldcg(a.logits + (int64_t)t * NE + e);
				__syncwarp();
				topk_token<LANES>(lg, a.router_bias, NE, K, a.mode_exact, a.renorm, sel,
						  reinterpret_cast<int32_t *>(sel + K), a.ids + (int64_t)t * K,
						  a.wts + (int64_t)t * K, nullptr, nullptr);
				if (shard) {
					// this token's ids into every rank's gathered ids: pair
					// (rank * T + t) * K + slot
					const int32_t *sid = reinterpret_cast<const int32_t *>(sel + K);
					for (int q = lane; q < a.world * K; q += 32) {
						const int r = q / K, sl = q - r * K;
						a.idg[r][kEpIdsHeader + ((int64_t)a.rank * T + t) * K + sl] = sid[sl];
					}
				}
			}
		}
		if (shard && blockIdx.x == 0 && tid < a.world)
			a.idg[tid][a.rank] = T;  // checked by every rank: the same T everywhere
		__syncthreads();
		stamp(a.stamps, kStTopk);
		if (shard) {
			// every CTA of every rank announces that its tokens and ids are
			// out (made visible system-wide, then one arrival per CTA on each
			// rank's counter for this rank); each rank waits for every rank's
			__threadfence_system();
			__syncthreads();
			if (tid == 0)
				for (int r = 0; r < a.world; r++)
					red_add_release_sys(a.routed[r] + kEpFlagStride * a.rank, 1ull);
			if (tid < a.world)
				wait_arrivals(a.routed[a.rank] + kEpFlagStride * tid, shard_epoch * gridDim.x,
					      ep_wait, a.err);
		} else if (tid == 0 && !local_topk) {
			grid_sync(a.gbar, a.err);
		}
		__syncthreads();
		stamp(a.stamps, kStB1b);
		// every CTA: the dispatch of all (token, slot) pairs (token-sharded:
		// every rank's) into its own shared memory.  The ids sit in the stage
		// ring behind the dispatch scratch until the experts start.
		int32_t *ds = reinterpret_cast<int32_t *>(smem);
		int np = T * K;
		const int32_t *idsrc = a.ids;
		if (shard) {
			const int32_t *hdr = a.idg[a.rank];
			bool same = true;
			for (int r = 0; r < a.world; r++)
				same = same && __ldcg(hdr + r) == T;
			if (!same && blockIdx.x == 0 && tid == 0)
				atomicCAS(a.err, 0, 5);  // an expired wait, recorded first, explains it
			np = same ? a.world * T * K : 0;
			idsrc = hdr + kEpIdsHeader;
		}
		if (!local_topk)
			for (int i = tid; i < np; i += blockDim.x)
				ids_all[i] = __ldcg(idsrc + i);
		for (int i = tid; i < T * K; i += blockDim.x)   // 1 / w, the combine's divisor
			wts_s[i] = __fdiv_rn(1.0f, local_topk ? wtok[i] : __ldcg(a.wts + i));
		__syncthreads();
		if (local_topk && np <= 32) {
			if (warp == 0)
				dispatch_warp(ids_all, np, NE, a.first_expert, a.n_local, counts_s, offsets_s,
					      perm_s, active_s, nact_s, a.err);
		} else {
			dispatch_body(ids_all, np, NE, a.first_expert, a.n_local, counts_s, offsets_s,
				      perm_s, nullptr, active_s, nact_s, a.err, ds);
		}
		__syncthreads();
		stamp(a.stamps, kStDispatch);
		const int n_active = *nact_s;
		for (int i = tid; i < n_active; i += blockDim.x) {
			const int e = active_s[i];
			en[i] = e | (counts_s[e] << 8);
			off[i] = offsets_s[e];
		}
		__syncthreads();
		if (warp == 0)
			build_prefix_warp(en, n_active, (F + 7) / 8, pre_gu);
		if (warp == 1)
			build_prefix_warp(en, n_active, (D + 16 * MT_DN - 1) / (16 * MT_DN), pre_dn);
		if (blockIdx.x == 0) {
			// the routing, for the host (moe_layer_routing)
			for (int i = tid; i < np; i += blockDim.x)
				a.perm[i] = perm_s[i];
			for (int i = tid; i < NE; i += blockDim.x) {
				a.counts[i] = counts_s[i];
				a.offsets[i] = offsets_s[i];
			}
			for (int i = tid; i < n_active; i += blockDim.x)
				a.active[i] = active_s[i];
			if (tid == 0) {
				a.offsets[NE] = offsets_s[NE];
				*a.n_active = n_active;
			}
		}
		__syncthreads();
	}
	stamp(a.stamps, kStP1);

	// ------------------------------------------------ P2, P3: experts
	{
		const int n_active = *nact_s;
		const Phase gu{a.dptrs, a.dptrs + NE, F, D, K, en, off, pre_gu, n_active, perm_s, 1, 0,
			       shard ? a.xg[a.rank] : a.x16, a.h16, nullptr, a.err, nullptr, nullptr, 0, 0};
		// down stores y per (token, slot) row: replicated tokens, here and
		// into every other rank's exchange buffer; token-sharded, into the
		// buffer of the rank that owns the token.  P4 divides by 1 / w and adds
		const Phase dn{a.dptrs + 2 * NE, nullptr, D, F, K, en, off, pre_dn, n_active, perm_s, 0, 1,
			       a.h16, nullptr, Y, a.err, nullptr, shard ? yall : ypeers,
			       (ep && !shard) ? a.world - 1 : 0, shard ? T * K : 0};
		Pipe pipe;
		if (warp == kProducerWarp) {
			core_producer<QT, true, STAGES, WB_GU>(gu, smem, b, pipe, lane);
			core_producer<QT, false, STAGES, WB_DN, MT_DN>(dn, smem, b, pipe, lane);
		} else {
			if (warp >= kEpiWarp0)
				core_epilogue<QT, true>(gu, red, stg + (warp - kEpiWarp0) * kEpiStage, b, pipe,
							warp - kEpiWarp0, lane);
			else if (D > WB_GU * kMmaWarps * QK)  // rows of several stages
				core_math<QT, true, STAGES, WB_GU, true, 1, true>(gu, smem, red, b, pipe, warp, lane);
			else
				core_math<QT, true, STAGES, WB_GU, true>(gu, smem, red, b, pipe, warp, lane);
			// every CTA's h rows must be written before any CTA reads them
			bar_math_epi();
			stamp(a.stamps, kStP2);
			if (tid == 0)
				grid_sync(a.gbar, a.err);
			bar_math_epi();
			stamp(a.stamps, kStB2);
			if (warp >= kEpiWarp0)
				core_epilogue<QT, false, MT_DN>(dn, red, stg + (warp - kEpiWarp0) * kEpiStage, b,
								pipe, warp - kEpiWarp0, lane);
			else if (F > WB_DN * (kMmaWarps / MT_DN) * QK)
				core_math<QT, false, STAGES, WB_DN, true, MT_DN, true>(dn, smem, red, b, pipe,
										warp, lane);
			else
				core_math<QT, false, STAGES, WB_DN, true, MT_DN>(dn, smem, red, b, pipe, warp,
									  lane);
		}
	}
	if (!ep) {
		__syncthreads();
		stamp(a.stamps, kStP3);
		if (tid == 0)
			grid_sync(a.gbar, a.err);
		__syncthreads();
	} else {
		// every CTA of every rank announces that its rows are out: the rows
		// it stored (here and over NVLink) are made visible system-wide,
		// then one arrival per CTA on each rank's counter for this rank;
		// each rank waits until every rank's CTAs have arrived
		__threadfence_system();
		__syncthreads();
		stamp(a.stamps, kStP3);
		if (tid == 0)
			for (int r = 0; r < a.world; r++)
				red_add_release_sys(a.inbound[r] + kEpFlagStride * a.rank, 1ull);
		if (tid < a.world)
			wait_arrivals(a.inbound[a.rank] + kEpFlagStride * tid, epoch * gridDim.x, ep_wait,
				      a.err);
		__syncthreads();
	}
	stamp(a.stamps, kStB3);

	// a kernel launched as a programmatic dependent of this one (the next
	// projection of a model's decode step) may start streaming its weights
	// on SMs this kernel leaves; it reads this layer's output only after
	// this grid completes
	griddep_launch_dependents();

	// ------------------------------------------------ P4: combine
	// one output element per thread; the rows of 8 slots are loaded before
	// their divisions, so the L2 round trips overlap
	{
		const int64_t total = (int64_t)T * D;
		for (int64_t i = (int64_t)blockIdx.x * blockDim.x + tid; i < total;
		     i += (int64_t)gridDim.x * blockDim.x) {
			const int t = (int)(i / D);
			const int j = (int)(i - (int64_t)t * D);
			const float *yt = Y + (int64_t)t * K * D + j;
			float acc = 0.0f;
			for (int s0 = 0; s0 < K; s0 += 8) {
				float y[8];
#pragma unroll
				for (int u = 0; u < 8; u++)
					y[u] = s0 + u < K ? __ldcg(yt + (int64_t)(s0 + u) * D) : 0.0f;
#pragma unroll
				for (int u = 0; u < 8; u++)
					if (s0 + u < K)
						acc = __fadd_rn(__fdiv_rn(y[u], wts_s[t * K + s0 + u]), acc);
			}
			a.out[(int64_t)t * D + j] = acc;
		}
	}
	stamp(a.stamps, kStEnd);
	if (ep && blockIdx.x == 0 && tid == 0) {
		*a.launches = epoch;  // every CTA read them before arriving above
		if (shard)
			*a.shard_launches = shard_epoch;
	}
}

// ---------------------------------------------------------------- launch
bool decode_supported(int qtype, int64_t T, int D, int F, int NE, int K, int64_t world_pairs,
		      uintptr_t x, uintptr_t router_w, uintptr_t out)
{
	const Shape dn = pick_shape(F, false);
	return (qtype == kQ8_0 || qtype == kQ4_0) && T >= 1 && T <= kDecodeMaxT &&
	       T * K <= kDecodeMaxPairs && world_pairs <= kDecodeMaxPairsAll && K >= 1 && K <= 32 && NE % 8 == 0 && NE <= kMaxActive &&
	       D % 2048 == 0 && dn.wb == 8 && x % 16 == 0 && router_w % 16 == 0 && out % 16 == 0;
}

int decode_stamps() { return kStamps; }

int decode_max_t() { return kDecodeMaxT; }

// stamp index ending each of the five reported stages (router, routing,
// gate/up, down, combine); stage 0 starts at the earliest kStStart
void decode_stage_ends(int *ends)
{
	const int e[5] = {kStP0, kStP1, kStP2, kStP3, kStEnd};
	for (int i = 0; i < 5; i++)
		ends[i] = e[i];
}

// MT_DN: m-tiles per down item (2 for d_ff = 1024, else 1)
template <int QT, int LANES, int MT_DN>
static cudaError_t launch_decode_t(const DecodeArgs &a, cudaStream_t st)
{
	constexpr int STAGES = QT == kQ8_0 ? 5 : 9;
	constexpr size_t smem = decode_smem_bytes<QT, STAGES>();
	static_assert(smem <= 227 * 1024, "fused decode kernel exceeds shared memory");
	static_assert(RTile<LANES>::BYTES <= STAGES * StageLayout<QT>::BYTES,
		      "the router tile fits in the stage ring");
	static_assert((2 + kCoreThreads / 32) * kMaxActive * 4 <= DecodeSmem::RING_IDS &&
			      (kCoreThreads / 32) * kLocalTopkBytes <= DecodeSmem::RING_IDS &&
			      DecodeSmem::RING_IDS + kDecodeMaxPairsAll * 4 + (kCoreThreads / 32) * 32 * 4 <=
				      STAGES * StageLayout<QT>::BYTES,
		      "the dispatch scratch and the pair ids fit in the stage ring");
	auto fn = moe_decode_kernel<QT, LANES, 8, 8, MT_DN, STAGES>;
	cudaError_t e = ensure_smem(fn, smem);
	if (e != cudaSuccess)
		return e;
	cudaLaunchConfig_t cfg = {};
	cfg.gridDim = dim3((unsigned)sm_count());
	cfg.blockDim = dim3(kCoreThreads);
	cfg.dynamicSmemBytes = smem;
	cfg.stream = st;
	cudaLaunchAttribute attr[1];
	attr[0].id = cudaLaunchAttributeCooperative;
	attr[0].val.cooperative = 1;
	cfg.attrs = attr;
	cfg.numAttrs = 1;
	return cudaLaunchKernelEx(&cfg, fn, a);
}

cudaError_t launch_decode_layer(const DecodeArgs &a, int qtype, int lanes, cudaStream_t st)
{
	const bool mt2 = pick_shape(a.F, false).mt == 2;
	const bool l16 = lanes != 8;
	if (qtype == kQ8_0) {
		if (mt2)
			return l16 ? launch_decode_t<kQ8_0, 16, 2>(a, st) : launch_decode_t<kQ8_0, 8, 2>(a, st);
		return l16 ? launch_decode_t<kQ8_0, 16, 1>(a, st) : launch_decode_t<kQ8_0, 8, 1>(a, st);
	}
	if (mt2)
		return l16 ? launch_decode_t<kQ4_0, 16, 2>(a, st) : launch_decode_t<kQ4_0, 8, 2>(a, st);
	return l16 ? launch_decode_t<kQ4_0, 16, 1>(a, st) : launch_decode_t<kQ4_0, 8, 1>(a, st);
}

}  // namespace moe
