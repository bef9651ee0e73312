// expert_mma.cu — stand-alone launch of the grouped expert pipeline
// (expert_core.cuh): one CTA per SM runs the producer, math and epilogue
// warps over the items of one matrix pass (gate/up with SwiGLU, or down),
// reading the routing tables that the dispatch kernel wrote.
#include "expert_core.cuh"
#include "kernels.h"

namespace moe {

template <int QT, bool DUAL, int STAGES, int WB, int MT>
__global__ void __launch_bounds__(kCoreThreads, 1) expert_mma_kernel(MmaArgs a)
{
	// WB = blocks per math warp per stage, MT = m-tiles per item (see
	// pick_shape); the launcher guarantees cols % KC == 0
	extern __shared__ __align__(128) uint8_t smem[];
	using SL = StageLayout<QT>;
	uint8_t *p = smem + STAGES * SL::BYTES;
	float4 *red = reinterpret_cast<float4 *>(p);                   // [kRedBufs][8][32]
	float *stg = reinterpret_cast<float *>(p + SL::RED);            // epilogue staging
	int32_t *en = reinterpret_cast<int32_t *>(p + SL::RED + SL::EPI);  // [256]
	int32_t *off = en + kMaxActive;                                 // [256]
	int32_t *pre = off + kMaxActive;                                // [257]
	uint64_t *bars = reinterpret_cast<uint64_t *>(pre + kMaxActive + 4);
	const Bars b = init_bars<STAGES>(bars);
	// routing tables of the active experts, read once per CTA
	const int n_active = *a.n_active;
	constexpr int ROWS = DUAL ? 8 : 16 * MT;
	const int groups = (a.rows + ROWS - 1) / ROWS;
	for (int i = threadIdx.x; i < n_active; i += blockDim.x) {
		const int e = a.active[i];
		en[i] = e | (a.counts[e] << 8);
		off[i] = a.offsets[e];
	}
	__syncthreads();
	if (threadIdx.x == 0)
		build_prefix(en, n_active, groups, pre);
	fence_mbar_init();
	__syncthreads();

	Phase ph{a.w1, a.w2, a.rows, a.cols, a.K, en, off, pre, n_active, a.perm, a.in_perm,
		 a.out_perm, a.in16, a.out16, a.out, a.err, nullptr, nullptr, 0};
	Pipe pipe;
	const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
	if (warp == kProducerWarp)
		core_producer<QT, DUAL, STAGES, WB, MT>(ph, smem, b, pipe, lane);
	else if (warp >= kEpiWarp0)
		core_epilogue<QT, DUAL, MT>(ph, red, stg + (warp - kEpiWarp0) * kEpiStage, b, pipe,
					    warp - kEpiWarp0, lane);
	else
		core_math<QT, DUAL, STAGES, WB, false, MT>(ph, smem, red, b, pipe, warp, lane);
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

template <int QT, bool DUAL, int STAGES, int WB, int MT>
static cudaError_t launch_t(const MmaArgs &a, cudaStream_t st)
{
	using SL = StageLayout<QT>;
	const size_t smem = (size_t)STAGES * SL::BYTES + SL::RED + SL::EPI +
			    (3 * kMaxActive + 4) * 4 +
			    (2 * STAGES + 2 * kRedBufs) * 8;
	auto fn = expert_mma_kernel<QT, DUAL, STAGES, WB, MT>;
	constexpr int threads = kCoreThreads;
	cudaError_t e = ensure_smem(fn, smem);
	if (e != cudaSuccess)
		return e;
	static int per_sm = 0;  // occupancy of this instantiation (the same on every B200)
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
	const int rows_per_item = DUAL ? 8 : 16 * MT;
	const int64_t max_items = (int64_t)a.n_local * ((a.rows + rows_per_item - 1) / rows_per_item);
	if (grid > max_items)
		grid = max_items;
	fn<<<(unsigned)grid, threads, smem, st>>>(a);
	return cudaGetLastError();
}

bool expert_mma_supported(int qtype, int cols)
{
	return (qtype == kQ8_0 || qtype == kQ4_0) && pick_shape(cols, true).wb > 0;
}

template <int QT, bool DUAL, int S>
static cudaError_t launch_wb(const MmaArgs &a, cudaStream_t st)
{
	const Shape sh = pick_shape(a.cols, DUAL);
	if (!DUAL && sh.mt == 2)
		return launch_t<QT, DUAL, S, 8, DUAL ? 1 : 2>(a, st);
	switch (sh.wb) {
	case 8: return launch_t<QT, DUAL, S, 8, 1>(a, st);
	case 4: return launch_t<QT, DUAL, S, 4, 1>(a, st);
	case 2: return launch_t<QT, DUAL, S, 2, 1>(a, st);
	case 1: return launch_t<QT, DUAL, S, 1, 1>(a, st);
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
