// noalloc.cu — moe_gemv_device_noalloc: the dense quantized GEMV with all of
// its scratch in a fixed device array, so that a call allocates nothing.
//
// Who needs it: callers that cannot call cudaMalloc (or any allocator) at
// the point of the call -- a real-time decode loop that must never pay
// cudaMalloc's implicit device synchronisation, or a host engine embedded in
// a process whose device memory budget is fixed and handed out by someone
// else, so that a library allocating behind its back breaks the budget.
// They pass inputs and outputs; the scratch lives in g_noalloc_scratch
// below, which every GPU that loads the library holds until exit.
//
// Scratch layout (kNoallocBytes = 1 MiB):
//   [0, 256)     launch metadata: expert pointer table, counts, offsets,
//                error flag, active list, work counter
//   [256, 1 MiB) fp16 hi/lo split of x: m * 2 * cols halves
// so m * cols <= (1 MiB - 256) / 4 = 262080 elements.
//
// Every call rewrites the metadata and the split (the work counter starts at
// zero each call).  The error flag is sticky: a bounded wait that expires
// inside the tensor-core kernel sets it, and moe_sync() reports it (and
// clears it) after synchronising.  All calls share the one array: calls
// that overlap on the GPU (different streams, or host threads) race on it.
// The device address of the array is looked up once per device on that
// device's first call (cudaGetSymbolAddress), so make that first call
// before any stream capture.
#include "moe_b200.h"
#include "common.cuh"
#include "kernels.h"

#include <cstdio>

namespace moe {
// capi.cu: record a message for moe_last_error(); initialise the library
// on the current device if needed (creates its stream, allocates nothing);
// the library stream
void set_last_error(const char *msg);
int ensure_library();
cudaStream_t library_stream();
}  // namespace moe

namespace {

constexpr size_t kNoallocBytes = 1u << 20;
constexpr size_t kNoallocMeta = 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocBytes];

struct NoallocMeta {
	const void *w;          // expert pointer table of one "expert"
	int32_t counts[1];
	int32_t offsets[2];
	int32_t err[1];
	int32_t active[1];
	int32_t n_active[1];
	int32_t work[2];
};
static_assert(sizeof(NoallocMeta) <= kNoallocMeta, "metadata fits its slot");

uint8_t *g_scratch_dev[kMaxDevices];  // device address per device

int cuda_error(cudaError_t e, const char *what)
{
	char msg[200];
	snprintf(msg, sizeof(msg), "moe_gemv_device_noalloc: %s: %s", what, cudaGetErrorString(e));
	moe::set_last_error(msg);
	return MOE_ERR_CUDA;
}

// slot k of a Q4_0 block holds element q4_pick(k) (the order in which the
// tensor-core kernel pairs 4-bit codes)
__device__ __forceinline__ int q4_pick(int k)
{
	const int base = k & ~31, c = (k & 31) >> 3, j = k & 7;
	return base + 4 * c + 16 * ((j >> 1) & 1) + ((j >> 2) & 1) + 2 * (j & 1);
}

// metadata of the one-expert launch plus the hi/lo split of x
__global__ void noalloc_prep_kernel(const void *w, const float *__restrict__ x, int64_t m,
				    int cols, int q4, NoallocMeta *meta, __half *__restrict__ x16)
{
	if (blockIdx.x == 0 && threadIdx.x == 0) {
		meta->w = w;
		meta->counts[0] = (int32_t)m;
		meta->offsets[0] = 0;
		meta->offsets[1] = (int32_t)m;
		meta->active[0] = 0;
		meta->n_active[0] = 1;
		meta->work[0] = meta->work[1] = 0;
	}
	if (!x16)
		return;
	const int64_t total = m * cols;
	for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
	     i += (int64_t)gridDim.x * blockDim.x) {
		const int64_t r = i / cols;
		const int k = (int)(i - r * cols);
		const float v = x[r * cols + (q4 ? q4_pick(k) : k)];
		const __half h = __float2half_rn(v);
		x16[r * 2 * cols + k] = h;
		x16[r * 2 * cols + cols + k] = __float2half_rn(__fsub_rn(v, __half2float(h)));
	}
}

}  // namespace

extern "C" MOE_API int moe_gemv_device_noalloc(const void *w, int qtype, int64_t rows,
						int64_t cols, const float *x, int64_t m, float *y,
						void *stream)
{
	if ((qtype != MOE_Q8_0 && qtype != MOE_Q4_0) || cols <= 0 || cols % QK || rows <= 0 ||
	    m < 0 || !w || !x || !y || rows > INT32_MAX || cols > INT32_MAX) {
		moe::set_last_error("moe_gemv_device_noalloc: bad qtype, shape or null pointer");
		return MOE_ERR_INVALID;
	}
	if (m == 0)
		return MOE_OK;
	const size_t need = (size_t)m * 2 * (size_t)cols * sizeof(__half);
	if ((uint64_t)m > (uint64_t)(kNoallocBytes / 4) ||
	    need > kNoallocBytes - kNoallocMeta) {
		char msg[160];
		snprintf(msg, sizeof(msg),
			 "moe_gemv_device_noalloc: m*cols = %lld exceeds the fixed scratch "
			 "(at most %zu elements)",
			 (long long)(m * cols), (kNoallocBytes - kNoallocMeta) / 4);
		moe::set_last_error(msg);
		return MOE_ERR_INVALID;
	}
	int dev = 0;
	if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
		moe::set_last_error("moe_gemv_device_noalloc: no current CUDA device");
		return MOE_ERR_CUDA;
	}
	// a NULL stream means the library stream, which moe_init creates (a
	// stream, no memory) on first use
	if (!stream)
		if (int rc = moe::ensure_library())
			return rc;
	if (!g_scratch_dev[dev]) {
		// set-up, once per device, with that device current
		uint8_t *ptr = nullptr;
		cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void **>(&ptr),
						     g_noalloc_scratch);
		if (e != cudaSuccess || !ptr) {
			char msg[160];
			snprintf(msg, sizeof(msg), "moe_gemv_device_noalloc: cudaGetSymbolAddress: %s",
				 cudaGetErrorString(e));
			moe::set_last_error(msg);
			return MOE_ERR_CUDA;
		}
		g_scratch_dev[dev] = ptr;
	}
	uint8_t *base = g_scratch_dev[dev];
	NoallocMeta *meta = reinterpret_cast<NoallocMeta *>(base);
	__half *x16 = reinterpret_cast<__half *>(base + kNoallocMeta);
	// NULL = the library stream, as for moe_gemv_device
	cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : moe::library_stream();
	// one activation row: the single-row GEMV needs no scratch, only the
	// error flag
	if (m == 1 && moe::gemv1_supported(qtype, rows, cols, (uintptr_t)w, (uintptr_t)x,
					   (uintptr_t)y)) {
		if (cudaError_t e = moe::launch_gemv1(w, qtype, rows, cols, x, y, meta->err, st))
			return cuda_error(e, "single-row GEMV launch");
		return MOE_OK;
	}
	const bool mma = moe::expert_mma_supported(qtype, (int)cols) && (uintptr_t)w % 16 == 0;

	int64_t blocks = (m * cols + 255) / 256;
	if (blocks > 148 * 32)
		blocks = 148 * 32;
	noalloc_prep_kernel<<<(unsigned)blocks, 256, 0, st>>>(w, x, m, (int)cols,
							      qtype == MOE_Q4_0, meta,
							      mma ? x16 : nullptr);
	if (cudaError_t e = cudaGetLastError())
		return cuda_error(e, "prep launch");
	if (mma) {
		moe::MmaArgs a{};
		a.w1 = reinterpret_cast<const void *const *>(&meta->w);
		a.qtype = qtype;
		a.rows = (int)rows;
		a.cols = (int)cols;
		a.NE = 1;
		a.K = 1;
		a.first_expert = 0;
		a.n_local = 1;
		a.counts = meta->counts;
		a.offsets = meta->offsets;
		a.perm = nullptr;
		a.in_perm = a.out_perm = 0;
		a.in16 = x16;
		a.out = y;
		a.dual = 0;
		a.err = meta->err;
		a.active = meta->active;
		a.n_active = meta->n_active;
		a.work = meta->work;
		if (cudaError_t e = moe::launch_expert_mma(a, st))
			return cuda_error(e, "tensor-core GEMV launch");
		return MOE_OK;
	}
	moe::GemvArgs a{};
	a.w1 = reinterpret_cast<const void *const *>(&meta->w);
	a.qtype = qtype;
	a.rows = (int)rows;
	a.cols = (int)cols;
	a.NE = 1;
	a.K = 1;
	a.first_expert = 0;
	a.n_local = 1;
	a.counts = meta->counts;
	a.offsets = meta->offsets;
	a.perm = nullptr;
	a.in_perm = a.out_perm = 0;
	a.in = x;
	a.out = y;
	a.dual = 0;
	if (cudaError_t e = moe::launch_expert_gemv(a, st))
		return cuda_error(e, "GEMV launch");
	return MOE_OK;
}

namespace moe {
// moe_sync's check of the sticky error flag of this device's noalloc
// scratch (after the stream is idle): MOE_ERR_TIMEOUT once per expired wait
int noalloc_take_error()
{
	int dev = 0;
	if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices || !g_scratch_dev[dev])
		return MOE_OK;
	NoallocMeta *meta = reinterpret_cast<NoallocMeta *>(g_scratch_dev[dev]);
	int32_t err = 0;
	cudaError_t e = cudaMemcpy(&err, meta->err, 4, cudaMemcpyDeviceToHost);
	if (e != cudaSuccess)
		return cuda_error(e, "reading the error flag");
	if (!err)
		return MOE_OK;
	e = cudaMemset(meta->err, 0, 4);
	if (e == cudaSuccess)
		e = cudaDeviceSynchronize();
	if (e != cudaSuccess)
		return cuda_error(e, "clearing the error flag");
	set_last_error("moe_gemv_device_noalloc: a bounded wait of the tensor-core GEMV expired "
		       "(the output of that call is not valid)");
	return MOE_ERR_TIMEOUT;
}
}  // namespace moe
