// decode.cu — the whole MoE layer of a decode-sized batch (T <= 64 tokens)
// in one persistent kernel: one CTA per SM, launched cooperatively so that
// all CTAs are resident and can meet at grid-wide barriers.
//
// It computes what models/olmoe/olmoe.c:343-407 (and llama.c:393-457 with
// renormalisation) compute, phase by phase:
//
//   P0  router logits (matmul.c:91-131 lane order, exact) by tiles of
//       8 or 16 tokens x 8 experts spread over the CTAs, each tile staged
//       into shared memory by bulk copies; every CTA also writes its share
//       of the fp16 hi/lo split of x that the expert phases read.
//   --  grid barrier
//   P1  CTA t computes softmax + top-k (nn.c:221-308) of token t; grid
//       barrier; then every CTA reads the selected (token, slot) pairs and
//       computes their stable dispatch by expert into its own shared
//       memory (redundant, but cheaper than another barrier); CTA 0 writes
//       the dispatch to global memory for the host.  Meanwhile each CTA's
//       producer warp asks L2 for its first gate/up weights.
//   P2  gate/up + SwiGLU over (active expert, 8-row) items — the expert
//       pipeline of expert_core.cuh, writing h as fp16 hi/lo rows.
//   --  grid barrier among the math and epilogue warps.  The producer warp
//       does not wait: down weights do not depend on h, so it keeps
//       streaming them into the stage ring while P2 drains elsewhere.
//   P3  down over (active expert, 16-row) items, writing one fp32 row per
//       (token, slot) pair.
//   --  grid barrier
//   P4  combine: out[t] = sum_s y[t,s] / (1/w[t,s]) in slot order
//       (olmoe.c:397-404); the divisions happen in P3's epilogue, P4 adds
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

// router tile of P0.  Threads 0-255 compute: warp w owns expert e0 + w of
// the tile, lane = (token tk, lane quad lq); each thread keeps LANES/4
// consecutive SIMD lanes of one (token, expert) logit.
template <int LANES>
struct RTile {
	static constexpr int LQ = LANES / 4;                 // lane quads per logit
	static constexpr int RT = 32 / LQ;                   // tokens per tile: 8 or 16
	static constexpr int RE = 8;                         // experts per tile
	static constexpr int CH = 512;                       // columns per chunk
	// row stride chosen so that the tokens of a quarter warp hit distinct banks
	static constexpr int RS = CH * 4 + (LANES == 16 ? 64 : 32);
	static constexpr int SLOT = (RT + RE) * RS;
	// chunks in flight: all four of a 2048-column row for 16 lanes (one
	// round trip per tile); three for the taller 8-lane tile
	static constexpr int NSLOT = LANES == 16 ? 4 : 3;
};

constexpr int kDecodeMaxT = 64;
constexpr int kPrefetchItems = 8;  // gate/up items per CTA hinted into L2 at start
constexpr int kDecodeMaxPairs = 1024;
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
	static constexpr int IDS = PRE_DN + (kMaxActive + 4) * 4;  // int32 [1024]
	static constexpr int WTS = IDS + kDecodeMaxPairs * 4;      // f32   [1024]
	static constexpr int PERM = WTS + kDecodeMaxPairs * 4;     // int32 [1024]
	static constexpr int COUNTS = PERM + kDecodeMaxPairs * 4;  // int32 [256]
	static constexpr int OFFSETS = COUNTS + kMaxActive * 4;    // int32 [260]
	static constexpr int ACTIVE = OFFSETS + (kMaxActive + 4) * 4;  // int32 [256]
	static constexpr int NACT = ACTIVE + kMaxActive * 4;       // int32 [4]
	static constexpr int BARS = NACT + 16;                     // u64 bars
	static constexpr int END = BARS;                           // + bars
};

template <int QT, int STAGES>
constexpr size_t decode_smem_bytes()
{
	return (size_t)STAGES * StageLayout<QT>::BYTES + StageLayout<QT>::RED +
	       StageLayout<QT>::SSUM + DecodeSmem::END +
	       (2 * STAGES + 2 * kRedBufs + 4) * 8;  // + up to 4 router slot barriers
}

// ---------------------------------------------------------------- grid barrier
__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long *p)
{
	unsigned long long v;
	asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
	return v;
}

// Called by one thread per CTA after a CTA-level barrier.  *ctr counts the
// arrivals since it was zeroed and is a multiple of gridDim.x between
// barriers, so an arrival's ticket tells which barrier it belongs to and the
// count that releases it: one atomic per CTA, then a bounded poll.
__device__ bool grid_sync(unsigned long long *ctr, int32_t *err)
{
	__threadfence();
	const unsigned long long n = gridDim.x;
	const unsigned long long ticket = atomicAdd(ctr, 1ull);
	const unsigned long long target = (ticket / n + 1) * n;
	if (ticket + 1 < target) {
		const uint64_t t0 = global_ns();
		while (ld_acquire_gpu(ctr) < target) {
			if (global_ns() - t0 > kWaitLimitNs) {
				atomicExch(err, 3);
				return false;
			}
			__nanosleep(32);
		}
	}
	__threadfence();
	return true;
}

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
__device__ void router_tiles(const DecodeArgs &a, uint8_t *slots, uint64_t *rbar)
{
	using R = RTile<LANES>;
	const int tid = threadIdx.x;
	const int n_tt = (a.T + R::RT - 1) / R::RT, n_et = a.NE / R::RE;
	const int nch = a.D / R::CH;
	const int lq = tid % R::LQ, tk = (tid % 32) / R::LQ, ek = tid / 32;  // for tid < 256
	uint32_t q = 0;  // chunks consumed by this CTA (slot use sequence)
	bool failed = false;
	for (int u = blockIdx.x; u < n_tt * n_et; u += gridDim.x) {
		const int t0 = (u / n_et) * R::RT, e0 = (u % n_et) * R::RE;
		const int nt = min(R::RT, a.T - t0);
		auto issue = [&](int c, uint32_t qq) {
			const int s = qq % R::NSLOT;
			uint8_t *base = slots + s * R::SLOT;
			mbar_arrive_expect_tx(&rbar[s], (uint32_t)((nt + R::RE) * R::CH * 4));
			for (int r = 0; r < nt; r++)
				bulk_g2s(base + r * R::RS, a.x + (int64_t)(t0 + r) * a.D + c * R::CH,
					 R::CH * 4, &rbar[s]);
			for (int r = 0; r < R::RE; r++)
				bulk_g2s(base + (R::RT + r) * R::RS,
					 a.router_w + (int64_t)(e0 + r) * a.D + c * R::CH, R::CH * 4, &rbar[s]);
		};
		if (tid == 0 && !failed) {
			fence_proxy_async();
			for (int c = 0; c < min(nch, R::NSLOT); c++)
				issue(c, q + c);
		}
		float acc[4] = {0.f, 0.f, 0.f, 0.f};
		for (int c = 0; c < nch; c++) {
			const uint32_t qq = q + c;
			const int s = qq % R::NSLOT;
			if (!failed && !mbar_wait(&rbar[s], (qq / R::NSLOT) & 1)) {
				failed = true;
				atomicExch(a.err, 2);
			}
			if (tid < 256 && !failed) {
				const float *xs = reinterpret_cast<const float *>(slots + s * R::SLOT + tk * R::RS);
				const float *ws =
					reinterpret_cast<const float *>(slots + s * R::SLOT + (R::RT + ek) * R::RS);
#pragma unroll 8
				for (int st = 0; st < R::CH / LANES; st++) {
					const int col = st * LANES + lq * 4;
					const float4 xv = *reinterpret_cast<const float4 *>(xs + col);
					const float4 wv = *reinterpret_cast<const float4 *>(ws + col);
					acc[0] = __fmaf_rn(xv.x, wv.x, acc[0]);
					acc[1] = __fmaf_rn(xv.y, wv.y, acc[1]);
					acc[2] = __fmaf_rn(xv.z, wv.z, acc[2]);
					acc[3] = __fmaf_rn(xv.w, wv.w, acc[3]);
				}
			}
			__syncthreads();  // the slot is free again
			if (tid == 0 && !failed && c + R::NSLOT < nch) {
				fence_proxy_async();
				issue(c + R::NSLOT, qq + R::NSLOT);
			}
		}
		q += nch;
		if (tid < 256) {
			// lane tree of the reference (upper half onto lower half); quads
			// live in consecutive threads
			if (R::LQ == 4) {
#pragma unroll
				for (int j = 0; j < 4; j++)
					acc[j] = __fadd_rn(acc[j], __shfl_down_sync(0xffffffffu, acc[j], 2, 4));
			}
#pragma unroll
			for (int j = 0; j < 4; j++)
				acc[j] = __fadd_rn(acc[j], __shfl_down_sync(0xffffffffu, acc[j], 1, R::LQ));
			const float sum = __fadd_rn(__fadd_rn(acc[0], acc[2]), __fadd_rn(acc[1], acc[3]));
			if (lq == 0 && tk < nt)
				a.logits[(int64_t)(t0 + tk) * a.NE + e0 + ek] = __fadd_rn(0.0f, sum);
		}
	}
}

// Ask L2 for the head of the gate/up items this CTA will most likely stream
// in P2 (the item range it would get if every expert had one pass of
// tokens), so that HBM works during the latency-bound routing instead of
// idling.  One warp; issued after the router's own loads are done, so that
// it does not queue in front of them.
template <int QT>
__device__ void prefetch_gate_up(const DecodeArgs &a, int lane)
{
	constexpr int BB = StageLayout<QT>::BB;
	const int groups = a.F / 8;
	const int64_t total = (int64_t)a.NE * groups;
	const int64_t i0 = total * blockIdx.x / gridDim.x;
	const int64_t i1 = min(total * (blockIdx.x + 1) / gridDim.x, i0 + kPrefetchItems);
	const uint32_t rb = (uint32_t)(a.D / QK * BB);
	for (int64_t it = i0; it < i1; it++) {
		const int e = (int)(it / groups), r = (int)(it % groups) * 8 + (lane & 7);
		if (lane < 16) {
			const uint8_t *w = static_cast<const uint8_t *>(a.dptrs[(lane < 8 ? 0 : a.NE) + e]);
			bulk_prefetch_l2(w + (int64_t)r * rb, rb);
		}
	}
}

// ---------------------------------------------------------------- the kernel
template <int QT, int LANES, int WB_GU, int WB_DN, int STAGES>
__global__ void __launch_bounds__(kCoreThreads, 1) moe_decode_kernel(DecodeArgs a)
{
	extern __shared__ __align__(128) uint8_t smem[];
	using SL = StageLayout<QT>;
	using DS = DecodeSmem;
	uint8_t *tail = smem + STAGES * SL::BYTES;
	float4 *red = reinterpret_cast<float4 *>(tail);
	float *ssum = reinterpret_cast<float *>(tail + SL::RED);
	uint8_t *tb = tail + SL::RED + SL::SSUM;
	int32_t *en = reinterpret_cast<int32_t *>(tb + DS::EN);
	int32_t *off = reinterpret_cast<int32_t *>(tb + DS::OFF);
	int32_t *pre_gu = reinterpret_cast<int32_t *>(tb + DS::PRE_GU);
	int32_t *pre_dn = reinterpret_cast<int32_t *>(tb + DS::PRE_DN);
	int32_t *ids_s = reinterpret_cast<int32_t *>(tb + DS::IDS);
	float *wts_s = reinterpret_cast<float *>(tb + DS::WTS);
	int32_t *perm_s = reinterpret_cast<int32_t *>(tb + DS::PERM);
	int32_t *counts_s = reinterpret_cast<int32_t *>(tb + DS::COUNTS);
	int32_t *offsets_s = reinterpret_cast<int32_t *>(tb + DS::OFFSETS);
	int32_t *active_s = reinterpret_cast<int32_t *>(tb + DS::ACTIVE);
	int32_t *nact_s = reinterpret_cast<int32_t *>(tb + DS::NACT);
	uint64_t *bars = reinterpret_cast<uint64_t *>(tb + DS::BARS);
	uint64_t *rbar = bars + 2 * STAGES + 2 * kRedBufs;  // [NSLOT] router slots

	const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
	const int T = a.T, D = a.D, F = a.F, NE = a.NE, K = a.K;
	stamp(a.stamps, kStStart);
	if (blockIdx.x == 0 && tid == 0)
		*a.err = 0;
	const Bars b = init_bars<STAGES>(bars);
	if (tid < RTile<LANES>::NSLOT)
		mbar_init(&rbar[tid], 1);
	fence_mbar_init();
	__syncthreads();

	// ------------------------------------------------ P0: logits + x split
	router_tiles<LANES>(a, smem, rbar);
	{
		const int64_t total = (int64_t)T * D;
		for (int64_t i = (int64_t)blockIdx.x * blockDim.x + tid; i < total;
		     i += (int64_t)gridDim.x * blockDim.x) {
			const int64_t r = i / D;
			const int k = (int)(i - r * D);
			const float v = __ldg(a.x + r * D + (QT == kQ4_0 ? q4_src(k) : k));
			const __half h = __float2half_rn(v);
			a.x16[r * 2 * D + k] = h;
			a.x16[r * 2 * D + D + k] = __float2half_rn(__fsub_rn(v, __half2float(h)));
		}
	}
	__syncthreads();
	stamp(a.stamps, kStP0);
	if (tid == 0)
		grid_sync(a.gbar, a.err);
	__syncthreads();
	stamp(a.stamps, kStB1);

	// ------------------------------------------------ P1: routing
	// softmax + top-k of token t by warp 0 of CTA t (t < T); the others
	// start the L2 prefetch of their first gate/up items
	{
		float *lg = reinterpret_cast<float *>(smem);                 // [NE]
		float *sel = lg + kMaxActive;                                // [2K]
		if (warp == kProducerWarp)
			prefetch_gate_up<QT>(a, lane);
		for (int t = blockIdx.x; t < T; t += gridDim.x) {
			if (warp == 0) {
				for (int e = lane; e < NE; e += 32)
					lg[e] = __ldcg(a.logits + (int64_t)t * NE + e);
				__syncwarp();
				topk_token<LANES>(lg, a.router_bias, NE, K, a.mode_exact, a.renorm, sel,
						  reinterpret_cast<int32_t *>(sel + K), a.ids + (int64_t)t * K,
						  a.wts + (int64_t)t * K, nullptr, nullptr);
			}
		}
		__syncthreads();
		stamp(a.stamps, kStTopk);
		if (tid == 0)
			grid_sync(a.gbar, a.err);
		__syncthreads();
		stamp(a.stamps, kStB1b);
		// every CTA: the dispatch of all (token, slot) pairs, in shared memory
		int32_t *ds = reinterpret_cast<int32_t *>(smem);
		for (int i = tid; i < T * K; i += blockDim.x) {
			ids_s[i] = __ldcg(a.ids + i);
			wts_s[i] = __ldcg(a.wts + i);
		}
		__syncthreads();
		dispatch_body(ids_s, T * K, NE, 0, NE, counts_s, offsets_s, perm_s, nullptr, active_s,
			      nact_s, a.err, ds);
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
			build_prefix_warp(en, n_active, (D + 15) / 16, pre_dn);
		if (blockIdx.x == 0) {
			// the routing, for the host (moe_layer_routing)
			for (int i = tid; i < T * K; i += blockDim.x)
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
			       a.x16, a.h16, nullptr, a.err, nullptr};
		// down stores z = y / (1 / w) per (token, slot) row; P4 only adds
		const Phase dn{a.dptrs + 2 * NE, nullptr, D, F, K, en, off, pre_dn, n_active, perm_s, 0, 1,
			       a.h16, nullptr, a.Y, a.err, wts_s};
		Pipe pipe;
		if (warp == kProducerWarp) {
			core_producer<QT, true, STAGES, WB_GU>(gu, smem, b, pipe, lane);
			core_producer<QT, false, STAGES, WB_DN>(dn, smem, b, pipe, lane);
		} else {
			if (warp >= kEpiWarp0)
				core_epilogue<QT, true>(gu, red, b, pipe, warp - kEpiWarp0, lane);
			else
				core_math<QT, true, STAGES, WB_GU, true>(gu, smem, red, ssum, b, pipe, warp, lane);
			// every CTA's h rows must be written before any CTA reads them
			bar_math_epi();
			stamp(a.stamps, kStP2);
			if (tid == 0)
				grid_sync(a.gbar, a.err);
			bar_math_epi();
			stamp(a.stamps, kStB2);
			if (warp >= kEpiWarp0)
				core_epilogue<QT, false>(dn, red, b, pipe, warp - kEpiWarp0, lane);
			else
				core_math<QT, false, STAGES, WB_DN, true>(dn, smem, red, ssum, b, pipe, warp, lane);
		}
	}
	__syncthreads();
	stamp(a.stamps, kStP3);
	if (tid == 0)
		grid_sync(a.gbar, a.err);
	__syncthreads();
	stamp(a.stamps, kStB3);

	// ------------------------------------------------ P4: combine
	{
		const int d4 = D / 4;
		const int64_t total = (int64_t)T * d4;
		for (int64_t i = (int64_t)blockIdx.x * blockDim.x + tid; i < total;
		     i += (int64_t)gridDim.x * blockDim.x) {
			const int t = (int)(i / d4);
			const int j4 = (int)(i - (int64_t)t * d4);
			float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
			for (int s = 0; s < K; s++) {
				const float4 z = __ldcg(reinterpret_cast<const float4 *>(
							       a.Y + ((int64_t)t * K + s) * D) + j4);
				acc.x = __fadd_rn(z.x, acc.x);
				acc.y = __fadd_rn(z.y, acc.y);
				acc.z = __fadd_rn(z.z, acc.z);
				acc.w = __fadd_rn(z.w, acc.w);
			}
			reinterpret_cast<float4 *>(a.out + (int64_t)t * D)[j4] = acc;
		}
	}
	stamp(a.stamps, kStEnd);
}

// ---------------------------------------------------------------- launch
bool decode_supported(int qtype, int64_t T, int D, int F, int NE, int K, uintptr_t x,
		      uintptr_t router_w, uintptr_t out)
{
	const int wb_dn = pick_wb(F);
	return (qtype == kQ8_0 || qtype == kQ4_0) && T >= 1 && T <= kDecodeMaxT &&
	       T * K <= kDecodeMaxPairs && K >= 1 && K <= 32 && NE % 8 == 0 && NE <= kMaxActive &&
	       D % 2048 == 0 && (wb_dn == 8 || wb_dn == 4) && x % 16 == 0 && router_w % 16 == 0 &&
	       out % 16 == 0;
}

int decode_stamps() { return kStamps; }

// stamp index ending each of the five reported stages (router, routing,
// gate/up, down, combine); stage 0 starts at the earliest kStStart
void decode_stage_ends(int *ends)
{
	const int e[5] = {kStP0, kStP1, kStP2, kStP3, kStEnd};
	for (int i = 0; i < 5; i++)
		ends[i] = e[i];
}

template <int QT, int LANES, int WB_DN>
static cudaError_t launch_decode_t(const DecodeArgs &a, cudaStream_t st)
{
	constexpr int STAGES = QT == kQ8_0 ? 5 : 9;
	constexpr size_t smem = decode_smem_bytes<QT, STAGES>();
	static_assert(smem <= 227 * 1024, "fused decode kernel exceeds shared memory");
	static_assert(RTile<LANES>::NSLOT * RTile<LANES>::SLOT <= STAGES * StageLayout<QT>::BYTES,
		      "router slots fit in the stage ring");
	auto fn = moe_decode_kernel<QT, LANES, 8, WB_DN, STAGES>;
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
	const int wb_dn = pick_wb(a.F);
	const bool l16 = lanes != 8;
	if (qtype == kQ8_0) {
		if (wb_dn == 8)
			return l16 ? launch_decode_t<kQ8_0, 16, 8>(a, st) : launch_decode_t<kQ8_0, 8, 8>(a, st);
		return l16 ? launch_decode_t<kQ8_0, 16, 4>(a, st) : launch_decode_t<kQ8_0, 8, 4>(a, st);
	}
	if (wb_dn == 8)
		return l16 ? launch_decode_t<kQ4_0, 16, 8>(a, st) : launch_decode_t<kQ4_0, 8, 8>(a, st);
	return l16 ? launch_decode_t<kQ4_0, 16, 4>(a, st) : launch_decode_t<kQ4_0, 8, 4>(a, st);
}

}  // namespace moe
