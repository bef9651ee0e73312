// capi.cu — the C ABI of libmoe_b200.so (declared in include/moe_b200.h).
//
// Host-side runtime: one CUDA stream per process, a weight registry that
// keeps each uploaded tensor's GGUF bytes resident in HBM keyed by its
// host address, cached layer objects for the tensor_t entry points, and a
// grow-only scratch arena per layer.  Every entry point validates shapes,
// returns a moe_status and records a message for moe_last_error().
#include "moe_b200.h"
#include "common.cuh"
#include "kernels.h"

#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <array>
#include <map>
#include <string>
#include <vector>

#ifndef MOE_B200_VERSION
#define MOE_B200_VERSION "moe_b200 0.1 sm_100a"
#endif

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...)
{
	char buf[512];
	va_list ap;
	va_start(ap, fmt);
	vsnprintf(buf, sizeof(buf), fmt, ap);
	va_end(ap);
	g_err = buf;
	return code;
}

int cuda_fail(cudaError_t e, const char *what)
{
	return fail(e == cudaErrorMemoryAllocation ? MOE_ERR_NOMEM : MOE_ERR_CUDA, "%s: %s", what,
		    cudaGetErrorString(e));
}

#define CK(call)                                                   \
	do {                                                       \
		cudaError_t e_ = (call);                           \
		if (e_ != cudaSuccess)                             \
			return cuda_fail(e_, #call);               \
	} while (0)

struct Reg {
	uintptr_t host;
	size_t bytes;
	void *dev;
};

struct Ctx {
	bool init = false;
	int device = -1;
	cudaStream_t stream = nullptr;
	std::map<uintptr_t, Reg> regs;  // keyed by host start address
	size_t resident = 0;
	// host-IO staging for the drop-ins
	void *pin = nullptr;
	size_t pin_bytes = 0;
	void *dev_io = nullptr;
	size_t dev_io_bytes = 0;
	int32_t *err_pin = nullptr;  // pinned word: a layer's error word read with the output
	int32_t *gemv_err = nullptr; // device error word of the single-row GEMV (moe_sync reads it)
	std::map<std::vector<uintptr_t>, moe_layer *> layers;
	// moe_ffn_forward's repeat calls: (router, gate, up, down host bases,
	// qtype, experts, d_ff, d_model, top-k) -> the layer in `layers`
	std::map<std::array<uintptr_t, 9>, moe_layer *> ffn_fast;
};

Ctx g;

// Destroy the cached layers whose key points into [host, host + bytes) (their
// device weights are about to be freed); the repeat-call map only refers to
// cached layers, so it is emptied.
void drop_layers_in(uintptr_t host, size_t bytes)
{
	g.ffn_fast.clear();
	for (auto lt = g.layers.begin(); lt != g.layers.end();) {
		bool hit = false;
		for (uintptr_t k : lt->first)
			hit |= k >= host && k < host + bytes;
		if (hit) {
			moe_layer_destroy(lt->second);
			lt = g.layers.erase(lt);
		} else {
			++lt;
		}
	}
}

// NCCL, loaded at run time (no link dependency): the expert-parallel
// communicator of larger batches.  dlopen by soname reuses a libnccl.so.2
// the process has already loaded (e.g. by a framework).
struct Nccl {
	void *lib = nullptr;
	ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
	ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
	ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t,
				   ncclComm_t, cudaStream_t) = nullptr;
	ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
				   cudaStream_t) = nullptr;
	ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t,
			     cudaStream_t) = nullptr;
	ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
	ncclResult_t (*group_start)() = nullptr;
	ncclResult_t (*group_end)() = nullptr;
	ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
	const char *(*error_string)(ncclResult_t) = nullptr;
	ncclComm_t comm = nullptr;
	int rank = 0, world = 1;
};

Nccl nccl;

int nccl_load()
{
	if (nccl.lib)
		return MOE_OK;
	void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
	if (!h)
		h = dlopen("libnccl.so.2", RTLD_NOW);
	if (!h)
		return fail(MOE_ERR_COMM, "libnccl.so.2 not found: %s", dlerror());
	nccl.get_unique_id = (decltype(nccl.get_unique_id))dlsym(h, "ncclGetUniqueId");
	nccl.comm_init_rank = (decltype(nccl.comm_init_rank))dlsym(h, "ncclCommInitRank");
	nccl.all_reduce = (decltype(nccl.all_reduce))dlsym(h, "ncclAllReduce");
	nccl.comm_destroy = (decltype(nccl.comm_destroy))dlsym(h, "ncclCommDestroy");
	nccl.error_string = (decltype(nccl.error_string))dlsym(h, "ncclGetErrorString");
	nccl.all_gather = (decltype(nccl.all_gather))dlsym(h, "ncclAllGather");
	nccl.send = (decltype(nccl.send))dlsym(h, "ncclSend");
	nccl.recv = (decltype(nccl.recv))dlsym(h, "ncclRecv");
	nccl.group_start = (decltype(nccl.group_start))dlsym(h, "ncclGroupStart");
	nccl.group_end = (decltype(nccl.group_end))dlsym(h, "ncclGroupEnd");
	if (!nccl.get_unique_id || !nccl.comm_init_rank || !nccl.all_reduce || !nccl.comm_destroy ||
	    !nccl.error_string || !nccl.all_gather || !nccl.send || !nccl.recv ||
	    !nccl.group_start || !nccl.group_end)
		return fail(MOE_ERR_COMM, "libnccl.so.2 lacks an entry point");
	nccl.lib = h;
	return MOE_OK;
}

#define CK_NCCL(call)                                                              \
	do {                                                                       \
		ncclResult_t r_ = (call);                                          \
		if (r_ != ncclSuccess)                                             \
			return fail(MOE_ERR_COMM, "%s: %s", #call, nccl.error_string(r_)); \
	} while (0)

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int64_t qrow_bytes(int type, int64_t cols)
{
	if (type == MOE_Q8_0)
		return cols / QK * Q8_0_BYTES;
	if (type == MOE_Q4_0)
		return cols / QK * Q4_0_BYTES;
	if (type == MOE_Q4_K)
		return cols / 256 * 144;
	if (type == MOE_Q6_K)
		return cols / 256 * 210;
	return cols * 4;
}

bool legacy_type(int t) { return t == MOE_Q8_0 || t == MOE_Q4_0; }
bool ktype(int t) { return t == MOE_Q4_K || t == MOE_Q6_K; }

// bytes of a tensor's payload from its dims (innermost dim = columns)
size_t tensor_bytes(const moe_tensor_t *t)
{
	if (t->ndim == 0)
		return 0;
	uint64_t cols = t->dim[t->ndim - 1];
	uint64_t rows = 1;
	for (uint32_t i = 0; i + 1 < t->ndim; i++)
		rows *= t->dim[i];
	return (size_t)(rows * (uint64_t)qrow_bytes(t->type, (int64_t)cols));
}

const void *tensor_host_ptr(const moe_tensor_t *t)
{
	return t->type == MOE_F32 ? (const void *)t->data : t->qdata;
}

// initialise on the current device (device 0 in a fresh process) if needed
int ensure_init()
{
	if (g.init)
		return MOE_OK;
	int dev = 0;
	if (cudaGetDevice(&dev) != cudaSuccess)
		dev = 0;
	return moe_init(dev) == MOE_OK ? MOE_OK : MOE_ERR_NOT_INIT;
}

// device address for host range [p, p+bytes): a registered range that
// contains it, else upload it now as a new registration.
int resolve(const void *hp, size_t bytes, const void **dev)
{
	uintptr_t p = (uintptr_t)hp;
	auto it = g.regs.upper_bound(p);
	if (it != g.regs.begin()) {
		--it;
		const Reg &r = it->second;
		if (p >= r.host && p + bytes <= r.host + r.bytes) {
			*dev = (const char *)r.dev + (p - r.host);
			return MOE_OK;
		}
	}
	// a registration at the same start that is too short is replaced
	auto same = g.regs.find(p);
	if (same != g.regs.end()) {
		CK(cudaDeviceSynchronize());
		drop_layers_in(same->second.host, same->second.bytes);
		cudaFree(same->second.dev);
		g.resident -= same->second.bytes;
		g.regs.erase(same);
	}
	void *d = nullptr;
	CK(cudaMalloc(&d, bytes));
	cudaError_t e = cudaMemcpy(d, hp, bytes, cudaMemcpyHostToDevice);
	if (e != cudaSuccess) {
		cudaFree(d);
		return cuda_fail(e, "weight upload");
	}
	g.regs[p] = Reg{p, bytes, d};
	g.resident += bytes;
	*dev = d;
	return MOE_OK;
}

int ensure_pinned(size_t bytes)
{
	if (g.pin_bytes >= bytes)
		return MOE_OK;
	if (g.pin)
		cudaFreeHost(g.pin);
	g.pin = nullptr;
	g.pin_bytes = 0;
	size_t want = align_up(bytes, 1 << 20);
	CK(cudaMallocHost(&g.pin, want));
	g.pin_bytes = want;
	return MOE_OK;
}

// the dense GEMV/GEMM error word (set by an expired bounded wait), read and
// cleared with the device idle
int take_gemv_error()
{
	if (!g.gemv_err)
		return MOE_OK;
	int32_t e = 0;
	CK(cudaMemcpy(&e, g.gemv_err, 4, cudaMemcpyDeviceToHost));
	if (!e)
		return MOE_OK;
	CK(cudaMemset(g.gemv_err, 0, 4));
	CK(cudaDeviceSynchronize());
	return fail(MOE_ERR_TIMEOUT, "moe_gemv_device: a bounded wait expired (the output of that "
		    "call is not valid)");
}

int ensure_dev_io(size_t bytes)
{
	if (!g.err_pin)
		CK(cudaHostAlloc(&g.err_pin, 64, cudaHostAllocDefault));
	if (g.dev_io_bytes >= bytes)
		return MOE_OK;
	CK(cudaStreamSynchronize(g.stream));
	if (g.dev_io)
		cudaFree(g.dev_io);
	g.dev_io = nullptr;
	g.dev_io_bytes = 0;
	size_t want = align_up(bytes, 1 << 20);
	CK(cudaMalloc(&g.dev_io, want));
	g.dev_io_bytes = want;
	return MOE_OK;
}

}  // namespace

namespace moe {
// used by noalloc.cu
void set_last_error(const char *msg) { g_err = msg ? msg : ""; }
int ensure_library()
{
	if (int rc = ensure_init())
		return rc;
	int dev = -1;
	cudaGetDevice(&dev);
	if (dev != g.device)
		return fail(MOE_ERR_INVALID, "the library stream belongs to device %d, the current "
			    "device is %d: pass a stream", g.device, dev);
	return MOE_OK;
}
cudaStream_t library_stream() { return g.init ? g.stream : nullptr; }
int noalloc_take_error();  // noalloc.cu
}  // namespace moe

// -------------------------------------------------------------------------
// layer object
// -------------------------------------------------------------------------
struct moe_layer {
	moe_layer_desc d;
	const void **dptrs = nullptr;  // device [3][NE]: gate, up, down
	void *scratch = nullptr;
	size_t scratch_bytes = 0;
	int64_t capT = -1;
	int64_t lastT = 0;
	int64_t last_pairs = 0;  // entries of perm written by the last forward
	// MOE_PROFILE: one set of 6 events per profiled forward since the last
	// moe_layer_stage_ms (stage boundaries on the launching stream)
	std::vector<std::array<cudaEvent_t, 6>> prof;
	std::vector<int> prof_fused;  // per record: 1 = fused kernel (phase stamps)
	size_t prof_used = 0;
	bool mma_ok = false;  // tensor-core kernels usable (cols % 256, 16 B aligned)
	bool gemm_ok = false; // prefill GEMM usable (weight tensor maps built)
	void *wmaps = nullptr;  // device [3][NE] weight tensor maps: gate, up, down
	// slices of scratch
	float *logits, *wts, *h, *Y;
	uint8_t *q8k = nullptr;    // K-quant experts: the tokens as Q8_K blocks
	int qt_gu = 0, qt_dn = 0;  // the experts' gate/up and down types
	__half *x16, *h16, *x16p;  // tokens hi/lo (token order), h hi/lo, tokens hi/lo (pair order)
	int32_t *ids, *counts, *offsets, *perm, *pos_of, *err;
	int32_t *active, *n_active, *work;  // [NE], [1], [2]
	unsigned long long *gbar;           // grid barrier arrivals of the fused kernel
	unsigned *t1cnt;                    // arrivals of the single-token router
	uint64_t *stamps;                   // [kStampRecords][grid][stamps]
	// expert parallelism (n_local < n_experts): exchange buffer of this rank
	// (moe::ep_layout: two Y halves, counters, gathered ids and tokens),
	// peers once connected
	char *xbuf = nullptr;
	int64_t y_half = 0;
	moe::EpLayout xl{};
	int ep_rank = 0, ep_world = 1;
	uint64_t ep_wait_ns = 0;            // 0: the kernel's default limit
	std::vector<void *> opened;         // peer buffers opened by IPC
	float **d_ybuf = nullptr;           // device [world]
	unsigned long long **d_inbound = nullptr, **d_routed = nullptr;
	__half **d_xg = nullptr;
	int32_t **d_idg = nullptr;
	// token-sharded forwards above the fused kernel's sizes (NCCL all-to-all)
	struct A2A {
		void *buf = nullptr;     // received tokens, their h and their rows
		size_t bytes = 0;
		int32_t *meta = nullptr; // device: every rank's counts, local counts,
		                         // offsets, active list, n_active
		int32_t *host = nullptr; // pinned mirror of meta
		size_t meta_ints = 0;
	} a2a;
};

namespace moe {
int64_t layer_scratch_rows(const moe_layer *L) { return L ? L->capT : -1; }
}  // namespace moe

namespace {

constexpr size_t kStampRecords = 64;  // profiled fused forwards kept per layer

// single-token layers of these expert types take the single-row GEMV path;
// MOE_T1=0 / MOE_T1=1 in the environment turn it off / on for both types
bool t1_on(int qtype)
{
	static const int mode = [] {
		const char *e = getenv("MOE_T1");
		return e ? (e[0] == '0' ? 0 : 1) : -1;
	}();
	if (mode >= 0)
		return mode == 1;
	return qtype == MOE_Q4_0;
}

int layer_scratch(moe_layer *L, int64_t T)
{
	if (T <= L->capT)
		return MOE_OK;
	const int64_t NE = L->d.n_experts, K = L->d.top_k, F = L->d.d_ff, D = L->d.d_model;
	const int64_t cap = T < 64 ? 64 : T;
	size_t off = 0;
	auto take = [&](size_t bytes) {
		size_t o = off;
		off = align_up(off + bytes, 256);
		return o;
	};
	size_t o_logits = take(cap * NE * 4), o_ids = take(cap * K * 4), o_wts = take(cap * K * 4);
	// token-sharded expert parallelism dispatches every rank's pairs
	const int64_t pcap = std::max<int64_t>(cap * K, L->xbuf ? moe::kDecodeMaxPairsAll : 0);
	size_t o_counts = take(NE * 4), o_offsets = take((NE + 1) * 4), o_perm = take(pcap * 4);
	size_t o_pos = take(cap * K * 4), o_err = take(4);
	size_t o_active = take(NE * 4), o_nact = take(4), o_work = take(8);
	size_t o_h = take((size_t)cap * K * F * 4), o_Y = take((size_t)cap * K * D * 4);
	size_t o_x16 = take((size_t)cap * 2 * D * 2), o_h16 = take((size_t)pcap * 2 * F * 2);
	size_t o_x16p = take((size_t)cap * K * 2 * D * 2);
	size_t o_q8k = take(D % 256 == 0 ? (size_t)cap * (D / 256) * 292 : 0);
	const size_t gbar_bytes = moe::decode_barrier_bytes(moe::sm_count());
	size_t o_gbar = take(gbar_bytes), o_t1cnt = take(4);
	size_t o_stamps = take((size_t)kStampRecords * moe::sm_count() * moe::decode_stamps() * 8);
	if (L->scratch) {
		CK(cudaStreamSynchronize(g.stream));
		cudaFree(L->scratch);
		L->scratch = nullptr;
		L->capT = -1;
	}
	CK(cudaMalloc(&L->scratch, off));
	L->scratch_bytes = off;
	char *b = static_cast<char *>(L->scratch);
	L->logits = (float *)(b + o_logits);
	L->ids = (int32_t *)(b + o_ids);
	L->wts = (float *)(b + o_wts);
	L->counts = (int32_t *)(b + o_counts);
	L->offsets = (int32_t *)(b + o_offsets);
	L->perm = (int32_t *)(b + o_perm);
	L->pos_of = (int32_t *)(b + o_pos);
	L->err = (int32_t *)(b + o_err);
	L->active = (int32_t *)(b + o_active);
	L->n_active = (int32_t *)(b + o_nact);
	L->work = (int32_t *)(b + o_work);
	L->h = (float *)(b + o_h);
	L->Y = (float *)(b + o_Y);
	L->x16 = (__half *)(b + o_x16);
	L->x16p = (__half *)(b + o_x16p);
	L->h16 = (__half *)(b + o_h16);
	L->q8k = (uint8_t *)(b + o_q8k);
	L->gbar = (unsigned long long *)(b + o_gbar);
	L->t1cnt = (unsigned *)(b + o_t1cnt);
	L->stamps = (uint64_t *)(b + o_stamps);
	CK(cudaMemset(L->gbar, 0, gbar_bytes));
	CK(cudaMemset(L->t1cnt, 0, 4));
	CK(cudaDeviceSynchronize());  // ordered before launches on any stream
	L->capT = cap;
	return MOE_OK;
}

// the status of a layer's device error word `err` (already read, with the
// device idle); clears the word, and after an expired wait the grid-barrier
// counter, so that the next forward starts clean
int take_error(moe_layer *L, int32_t err)
{
	if (err == 0)
		return MOE_OK;
	CK(cudaMemset(L->err, 0, 4));
	if (err == 2 || err == 3 || err == 4)
		CK(cudaMemset(L->gbar, 0, moe::decode_barrier_bytes(moe::sm_count())));
	CK(cudaDeviceSynchronize());
	switch (err) {
	case 1:
		return fail(MOE_ERR_INVALID, "dispatch saw an expert id out of range");
	case 2:
		return fail(MOE_ERR_TIMEOUT, "an expert kernel's bounded wait expired");
	case 3:
		return fail(MOE_ERR_TIMEOUT, "the fused layer kernel's grid barrier expired");
	case 4:
		return fail(MOE_ERR_TIMEOUT, "the expert-parallel exchange wait expired (a rank "
			    "missing or behind; every rank calls moe_layer_ep_reset before going on)");
	case 5:
		return fail(MOE_ERR_INVALID, "token-sharded forward: the ranks passed different T");
	default:
		return fail(MOE_ERR_CUDA, "layer error word %d", (int)err);
	}
}

// Token-sharded expert parallelism above the fused kernel's sizes: this
// rank routes its own T tokens over all experts; each pair's token row
// (fp16 hi/lo) travels to the rank that owns the pair's expert, every rank
// runs the grouped GEMMs over the pairs it received (grouped by expert), the
// rows travel back, and each rank combines its own tokens in slot order.
// The transfers are NCCL point-to-point operations in one group per
// direction (an all-to-all-v), one per (peer, expert) segment, so that the
// received rows land grouped by expert; the segment sizes come from an
// all-gather of every rank's per-expert counts, read on the host (one
// synchronisation of the stream per forward).
int forward_sharded_a2a(moe_layer *L, const float *x, float *out, int64_t T, int flags,
			cudaStream_t st, cudaEvent_t *ev)
{
	const moe_layer_desc &d = L->d;
	const int NE = (int)d.n_experts, K = (int)d.top_k, D = (int)d.d_model, F = (int)d.d_ff;
	const int world = nccl.world, rank = nccl.rank;
	auto range = [&](int r, int &f, int &n) {
		f = (int)((int64_t)r * NE / world);
		n = (int)((int64_t)(r + 1) * NE / world) - f;
	};
	int f0, n0;
	range(rank, f0, n0);
	if (!nccl.comm || world < 2 || f0 != d.first_expert || n0 != d.n_local)
		return fail(MOE_ERR_INVALID, "token-sharded forward of %lld tokens: needs moe_ep_init "
			    "and the layer to own experts [r*NE/world, (r+1)*NE/world)", (long long)T);
	if (!L->gemm_ok || (uintptr_t)x % 16)
		return fail(MOE_ERR_UNSUPPORTED, "token-sharded forward of %lld tokens: needs the "
			    "grouped GEMM (weights and x 16-byte aligned, shapes as it requires)",
			    (long long)T);
	cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
	CK(cudaStreamIsCapturing(st, &cap));
	if (cap != cudaStreamCaptureStatusNone)
		return fail(MOE_ERR_UNSUPPORTED, "token-sharded forward of %lld tokens reads the "
			    "transfer sizes on the host: it cannot be captured", (long long)T);
	const int lanes = (flags & MOE_LANES_AVX2) ? 8 : 16;
	const int q4 = d.qtype == MOE_Q4_0;
	const int mode_exact = (flags & MOE_TOPK_EXACT) ? 1 : 0, renorm = (flags & MOE_RENORM) ? 1 : 0;
	auto record = [&](int i) { return ev ? cudaEventRecord(ev[i], st) : cudaSuccess; };
	const int64_t P = T * K;
	// [0] router logits of this rank's tokens
	if (moe::router_tiled_ok(D, NE))
		CK(moe::launch_router_tiled(x, d.router_w, (int)T, D, NE, lanes, L->logits, nullptr, q4, st));
	else
		CK(moe::launch_router_logits(x, d.router_w, (int)T, D, NE, lanes, L->logits, st));
	CK(record(1));
	// [1] top-k and the dispatch of this rank's pairs over every expert
	if (T <= 256 && moe::route_small_smem((int)T, NE, K) <= 160 * 1024) {
		CK(moe::launch_route_small(L->logits, d.router_bias, (int)T, NE, K, lanes, mode_exact,
					   renorm, 0, NE, L->ids, L->wts, L->counts, L->offsets, L->perm,
					   L->pos_of, L->active, L->n_active, L->err, L->work, st));
	} else {
		CK(moe::launch_router_topk(L->logits, d.router_bias, (int)T, NE, K, lanes, mode_exact,
					   renorm, L->ids, L->wts, nullptr, st));
		CK(moe::launch_dispatch(L->ids, (int)P, NE, 0, NE, L->counts, L->offsets, L->perm,
					L->pos_of, L->active, L->n_active, L->err, L->work, st));
	}
	// this rank's pairs in expert order as fp16 hi/lo: the send buffer
	CK(moe::launch_gather_split(x, L->perm, P, D, K, L->x16p, st));
	// every rank's per-expert counts; local counts, offsets, active list,
	// n_active;
	// the segment table (up to NE segments of 3 int64)
	const size_t mi = (size_t)world * NE + 3 * (size_t)NE + 4 + 6 * (size_t)NE + 4;
	if (L->a2a.meta_ints < mi) {
		CK(cudaStreamSynchronize(st));
		cudaFree(L->a2a.meta);
		if (L->a2a.host)
			cudaFreeHost(L->a2a.host);
		L->a2a.meta = nullptr;
		L->a2a.host = nullptr;
		L->a2a.meta_ints = 0;
		CK(cudaMalloc(&L->a2a.meta, mi * 4));
		CK(cudaHostAlloc(&L->a2a.host, mi * 4, cudaHostAllocDefault));
		L->a2a.meta_ints = mi;
	}
	int32_t *allc_d = L->a2a.meta, *allc = L->a2a.host;
	CK_NCCL(nccl.all_gather(L->counts, allc_d, NE, ncclInt32, nccl.comm, st));
	CK(cudaMemcpyAsync(allc, allc_d, (size_t)world * NE * 4, cudaMemcpyDeviceToHost, st));
	CK(cudaStreamSynchronize(st));
	// the plan.  Own pairs are expert-sorted, so the pairs for rank r are
	// one contiguous range: one send per peer.  Rank q's pairs arrive as one
	// contiguous range per source (source-major: by source, then by local
	// expert), and a segment copy puts them expert-major (by local expert,
	// then by source), the order the grouped GEMM reads.  The rows go back
	// the same way reversed and land at the pairs' dispatch positions.
	const int32_t *own = allc + (size_t)rank * NE;
	std::vector<int64_t> o(NE + 1, 0);
	for (int e = 0; e < NE; e++)
		o[e + 1] = o[e] + own[e];
	int32_t *cnt_l = allc + (size_t)world * NE, *off_l = cnt_l + NE, *act = off_l + NE + 1;
	int32_t *nact = act + NE;
	int64_t pl = 0;
	int na = 0;
	std::vector<int64_t> rpos((size_t)world * NE, 0);  // [q][e]: expert-major start
	for (int e = 0; e < NE; e++) {
		off_l[e] = (int32_t)pl;
		int64_t c = 0;
		if (e >= f0 && e < f0 + n0)
			for (int q = 0; q < world; q++) {
				rpos[(size_t)q * NE + e] = pl + c;
				c += allc[(size_t)q * NE + e];
			}
		cnt_l[e] = (int32_t)c;
		if (c > 0)
			act[na++] = e;
		pl += c;
	}
	off_l[NE] = (int32_t)pl;
	*nact = na;
	if (pl > INT32_MAX / 2)
		return fail(MOE_ERR_INVALID, "token-sharded forward: %lld pairs for one rank", (long long)pl);
	// source-major starts and the segment table [nseg][3] = (source-major
	// row, expert-major row, rows)
	std::vector<int64_t> soff(world + 1, 0);
	const size_t seg_at = ((size_t)(nact - allc) + 2) & ~(size_t)1;  // even: 8-byte aligned
	int64_t *seg = reinterpret_cast<int64_t *>(allc + seg_at);
	int nseg = 0;
	for (int q = 0; q < world; q++) {
		int64_t c = soff[q];
		for (int e = f0; e < f0 + n0; e++) {
			const int32_t n = allc[(size_t)q * NE + e];
			if (n) {
				seg[3 * nseg] = c;
				seg[3 * nseg + 1] = rpos[(size_t)q * NE + e];
				seg[3 * nseg + 2] = n;
				nseg++;
			}
			c += n;
		}
		soff[q + 1] = c;
	}
	// receive-side buffers: tokens source-major and expert-major [pl][2][D],
	// h [pl][2][F] (fp16), rows expert-major and source-major [pl][D]
	const size_t bx = align_up((size_t)pl * 2 * D * 2, 256), bh = align_up((size_t)pl * 2 * F * 2, 256);
	const size_t by = align_up((size_t)pl * D * 4, 256);
	const size_t need = 2 * bx + bh + 2 * by + 256;
	if (need > L->a2a.bytes) {
		cudaFree(L->a2a.buf);
		L->a2a.buf = nullptr;
		L->a2a.bytes = 0;
		CK(cudaMalloc(&L->a2a.buf, need));
		L->a2a.bytes = need;
	}
	char *ab = (char *)L->a2a.buf;
	__half *xs = (__half *)ab, *xr = (__half *)(ab + bx), *hr = (__half *)(ab + 2 * bx);
	float *yr = (float *)(ab + 2 * bx + bh), *ys = (float *)(ab + 2 * bx + bh + by);
	const size_t meta_loc = (size_t)world * NE;
	const size_t meta_bytes = (size_t)((char *)(seg + 3 * nseg) - (char *)cnt_l);
	CK(cudaMemcpyAsync(allc_d + meta_loc, cnt_l, meta_bytes, cudaMemcpyHostToDevice, st));
	const int64_t *seg_d = reinterpret_cast<const int64_t *>(
		allc_d + meta_loc + ((int32_t *)seg - cnt_l));
	const size_t xrow = (size_t)2 * D;  // halves per token row
	int fr, nr;
	// [2] token rows to the experts' ranks (own experts: a device copy)
	CK(record(2));
	if (soff[rank + 1] > soff[rank])
		CK(cudaMemcpyAsync(xs + soff[rank] * xrow, L->x16p + o[f0] * xrow,
				   (size_t)(soff[rank + 1] - soff[rank]) * xrow * 2,
				   cudaMemcpyDeviceToDevice, st));
	CK_NCCL(nccl.group_start());
	for (int r = 0; r < world; r++) {
		if (r == rank)
			continue;
		range(r, fr, nr);
		if (o[fr + nr] > o[fr])
			CK_NCCL(nccl.send(L->x16p + o[fr] * xrow, (size_t)(o[fr + nr] - o[fr]) * xrow,
					  ncclFloat16, r, nccl.comm, st));
		if (soff[r + 1] > soff[r])
			CK_NCCL(nccl.recv(xs + soff[r] * xrow, (size_t)(soff[r + 1] - soff[r]) * xrow,
					  ncclFloat16, r, nccl.comm, st));
	}
	CK_NCCL(nccl.group_end());
	CK(moe::launch_copy_segments(xs, xr, seg_d, nseg, 0, (int64_t)xrow * 2, st));
	// [3] the grouped GEMMs over the received pairs
	const size_t mb = moe::weight_map_bytes();
	moe::GemmArgs gu{};
	gu.maps1 = L->wmaps;
	gu.maps2 = (const uint8_t *)L->wmaps + NE * mb;
	gu.qtype = d.qtype;
	gu.rows = F;
	gu.cols = D;
	gu.n_local = (int)d.n_local;
	gu.counts = allc_d + meta_loc;
	gu.offsets = gu.counts + NE;
	gu.perm = nullptr;
	gu.active = gu.offsets + NE + 1;
	gu.n_active = gu.active + NE;
	gu.out_perm = 0;
	gu.in16 = xr;
	gu.out16 = hr;
	gu.dual = 1;
	gu.err = L->err;
	CK(moe::launch_expert_gemm(gu, pl, st));
	CK(record(3));
	moe::GemmArgs dn = gu;
	dn.maps1 = (const uint8_t *)L->wmaps + 2 * NE * mb;
	dn.maps2 = nullptr;
	dn.rows = D;
	dn.cols = F;
	dn.in16 = hr;
	dn.out16 = nullptr;
	dn.out = yr;
	dn.dual = 0;
	CK(moe::launch_expert_gemm(dn, pl, st));
	CK(record(4));
	// [4] the rows back to the tokens' ranks, at the pairs' dispatch positions
	CK(moe::launch_copy_segments(yr, ys, seg_d, nseg, 1, (int64_t)D * 4, st));
	if (soff[rank + 1] > soff[rank])
		CK(cudaMemcpyAsync(L->Y + o[f0] * D, ys + soff[rank] * D,
				   (size_t)(soff[rank + 1] - soff[rank]) * D * 4, cudaMemcpyDeviceToDevice,
				   st));
	CK_NCCL(nccl.group_start());
	for (int r = 0; r < world; r++) {
		if (r == rank)
			continue;
		range(r, fr, nr);
		if (soff[r + 1] > soff[r])
			CK_NCCL(nccl.send(ys + soff[r] * D, (size_t)(soff[r + 1] - soff[r]) * D, ncclFloat32,
					  r, nccl.comm, st));
		if (o[fr + nr] > o[fr])
			CK_NCCL(nccl.recv(L->Y + o[fr] * D, (size_t)(o[fr + nr] - o[fr]) * D, ncclFloat32, r,
					  nccl.comm, st));
	}
	CK_NCCL(nccl.group_end());
	CK(moe::launch_combine_pos(L->Y, L->pos_of, L->wts, (int)T, K, D, out, st));
	CK(record(5));
	L->last_pairs = P;
	return MOE_OK;
}

}  // namespace

extern "C" {

int moe_init(int device)
{
	if (g.init) {
		if (device == g.device)
			return MOE_OK;
		return fail(MOE_ERR_INVALID, "moe_init: already initialised on device %d", g.device);
	}
	int n = 0;
	CK(cudaGetDeviceCount(&n));
	if (device < 0 || device >= n)
		return fail(MOE_ERR_INVALID, "moe_init: device %d of %d", device, n);
	CK(cudaSetDevice(device));
	CK(cudaStreamCreateWithFlags(&g.stream, cudaStreamNonBlocking));
	g.device = device;
	g.init = true;
	g_err.clear();
	return MOE_OK;
}

int moe_shutdown(void)
{
	if (!g.init)
		return MOE_OK;
	cudaStreamSynchronize(g.stream);
	moe_ep_finalize();
	for (auto &kv : g.layers)
		moe_layer_destroy(kv.second);
	g.layers.clear();
	g.ffn_fast.clear();
	for (auto &kv : g.regs)
		cudaFree(kv.second.dev);
	g.regs.clear();
	g.resident = 0;
	if (g.pin)
		cudaFreeHost(g.pin);
	if (g.err_pin)
		cudaFreeHost(g.err_pin);
	g.err_pin = nullptr;
	cudaFree(g.gemv_err);
	g.gemv_err = nullptr;
	if (g.dev_io)
		cudaFree(g.dev_io);
	g.pin = g.dev_io = nullptr;
	g.pin_bytes = g.dev_io_bytes = 0;
	cudaStreamDestroy(g.stream);
	g.stream = nullptr;
	g.init = false;
	g.device = -1;
	return MOE_OK;
}

int moe_ep_unique_id(void *id)
{
	if (!id)
		return fail(MOE_ERR_INVALID, "moe_ep_unique_id: null argument");
	if (int rc = nccl_load())
		return rc;
	ncclUniqueId u;
	CK_NCCL(nccl.get_unique_id(&u));
	memcpy(id, &u, sizeof(u));
	return MOE_OK;
}

int moe_ep_init(int rank, int world, const void *id)
{
	if (!id || world < 1 || rank < 0 || rank >= world)
		return fail(MOE_ERR_INVALID, "moe_ep_init: rank %d of %d", rank, world);
	if (int rc = ensure_init())
		return rc;
	if (int rc = nccl_load())
		return rc;
	if (nccl.comm)
		return fail(MOE_ERR_INVALID, "moe_ep_init: already initialised");
	ncclUniqueId u;
	memcpy(&u, id, sizeof(u));
	CK_NCCL(nccl.comm_init_rank(&nccl.comm, world, u, rank));
	nccl.rank = rank;
	nccl.world = world;
	return MOE_OK;
}

int moe_ep_finalize(void)
{
	if (!nccl.comm)
		return MOE_OK;
	if (g.init)
		cudaStreamSynchronize(g.stream);
	const ncclResult_t r = nccl.comm_destroy(nccl.comm);
	nccl.comm = nullptr;
	nccl.rank = 0;
	nccl.world = 1;
	if (r != ncclSuccess)
		return fail(MOE_ERR_COMM, "ncclCommDestroy: %s", nccl.error_string(r));
	return MOE_OK;
}

const char *moe_last_error(void) { return g_err.c_str(); }

const char *moe_version(void) { return MOE_B200_VERSION; }

int moe_sync(void)
{
	if (!g.init)
		return fail(MOE_ERR_NOT_INIT, "moe_sync: not initialised");
	CK(cudaStreamSynchronize(g.stream));
	if (int rc = take_gemv_error())
		return rc;
	return moe::noalloc_take_error();
}

// ---------------------------------------------------------------- registry
int moe_register_weights(const moe_tensor_t *t)
{
	if (!t || !tensor_host_ptr(t))
		return fail(MOE_ERR_INVALID, "moe_register_weights: null tensor");
	if (t->type != MOE_F32 && t->type != MOE_Q8_0 && t->type != MOE_Q4_0)
		return fail(MOE_ERR_UNSUPPORTED, "moe_register_weights: dtype %d", t->type);
	if (int rc = ensure_init())
		return rc;
	const void *dev;
	return resolve(tensor_host_ptr(t), tensor_bytes(t), &dev);
}

int moe_unregister_weights(const moe_tensor_t *t)
{
	if (!t || !g.init)
		return fail(MOE_ERR_INVALID, "moe_unregister_weights: nothing registered");
	auto it = g.regs.find((uintptr_t)tensor_host_ptr(t));
	if (it == g.regs.end())
		return fail(MOE_ERR_INVALID, "moe_unregister_weights: tensor not registered");
	CK(cudaStreamSynchronize(g.stream));
	drop_layers_in(it->second.host, it->second.bytes);
	cudaFree(it->second.dev);
	g.resident -= it->second.bytes;
	g.regs.erase(it);
	return MOE_OK;
}

size_t moe_resident_bytes(void) { return g.resident; }

// ---------------------------------------------------------------- memory
void *moe_device_alloc(size_t bytes)
{
	if (ensure_init())
		return nullptr;
	void *p = nullptr;
	cudaError_t e = cudaMalloc(&p, bytes ? bytes : 1);
	if (e != cudaSuccess) {
		cuda_fail(e, "moe_device_alloc");
		return nullptr;
	}
	return p;
}

int moe_device_free(void *p)
{
	if (p)
		CK(cudaFree(p));
	return MOE_OK;
}

int moe_memcpy_h2d(void *dst, const void *src, size_t bytes)
{
	CK(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
	return MOE_OK;
}

int moe_memcpy_d2h(void *dst, const void *src, size_t bytes)
{
	CK(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost));
	return MOE_OK;
}

void *moe_host_alloc(size_t bytes)
{
	if (ensure_init())
		return nullptr;
	void *p = nullptr;
	cudaError_t e = cudaMallocHost(&p, bytes ? bytes : 1);
	if (e != cudaSuccess) {
		cuda_fail(e, "moe_host_alloc");
		return nullptr;
	}
	return p;
}

int moe_host_free(void *p)
{
	if (p)
		CK(cudaFreeHost(p));
	return MOE_OK;
}

// ---------------------------------------------------------------- synth
int moe_synth_gauss(float *dst, uint64_t seed, uint64_t tag, uint64_t offset, int64_t n,
		    float sd, void *stream)
{
	if (int rc = ensure_init())
		return rc;
	// stream seed: mix64(mix64(seed) ^ tag * 0xD1B54A32D192ED03)
	auto mix = [](uint64_t z) {
		z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
		z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
		return z ^ (z >> 31);
	};
	uint64_t s = mix(mix(seed) ^ (tag * 0xD1B54A32D192ED03ULL));
	cudaStream_t st = stream ? (cudaStream_t)stream : g.stream;
	CK(moe::launch_synth_gauss(dst, s, offset, n, sd, st));
	return MOE_OK;
}

int moe_quantize_device(const float *src, int64_t rows, int64_t cols, int qtype, void *dst,
			void *stream)
{
	if (int rc = ensure_init())
		return rc;
	if ((qtype != MOE_Q8_0 && qtype != MOE_Q4_0) || cols % QK)
		return fail(MOE_ERR_INVALID, "moe_quantize_device: qtype %d cols %lld", qtype,
			    (long long)cols);
	cudaStream_t st = stream ? (cudaStream_t)stream : g.stream;
	CK(moe::launch_quantize(src, rows, cols, qtype, dst, st));
	return MOE_OK;
}

// ---------------------------------------------------------------- layers
int moe_layer_create(moe_layer **out, const moe_layer_desc *desc)
{
	if (!out || !desc)
		return fail(MOE_ERR_INVALID, "moe_layer_create: null argument");
	if (int rc = ensure_init())
		return rc;
	const moe_layer_desc &d = *desc;
	const int qt_gu = MOE_QTYPE_GU(d.qtype), qt_dn = MOE_QTYPE_DN(d.qtype);
	const bool kq = ktype(qt_gu) || ktype(qt_dn);
	if (!(kq ? (ktype(qt_gu) && ktype(qt_dn)) : (d.qtype == MOE_Q8_0 || d.qtype == MOE_Q4_0)))
		return fail(MOE_ERR_UNSUPPORTED, "moe_layer_create: qtype %d (Q8_0 / Q4_0, or Q4_K / "
			    "Q6_K for gate/up and down)", d.qtype);
	if (kq && (d.d_model % 256 || d.d_ff % 256))
		return fail(MOE_ERR_INVALID, "moe_layer_create: K-quant experts need d_model and d_ff "
			    "multiples of 256");
	if (d.d_model <= 0 || d.d_ff <= 0 || d.d_model % QK || d.d_ff % QK)
		return fail(MOE_ERR_INVALID, "moe_layer_create: d_model %lld / d_ff %lld must be "
			    "positive multiples of 32", (long long)d.d_model, (long long)d.d_ff);
	if (d.n_experts <= 0 || d.n_experts > 256 || d.top_k <= 0 || d.top_k > d.n_experts ||
	    d.top_k > 64)
		return fail(MOE_ERR_INVALID, "moe_layer_create: n_experts %lld top_k %lld",
			    (long long)d.n_experts, (long long)d.top_k);
	if (!d.router_w || !d.gate || !d.up || !d.down)
		return fail(MOE_ERR_INVALID, "moe_layer_create: missing weight pointers");
	int64_t first = d.first_expert, nl = d.n_local;
	if (nl == 0 && first == 0)
		nl = d.n_experts;
	if (first < 0 || nl <= 0 || first + nl > d.n_experts)
		return fail(MOE_ERR_INVALID, "moe_layer_create: experts [%lld, +%lld) of %lld",
			    (long long)first, (long long)nl, (long long)d.n_experts);
	for (int64_t e = first; e < first + nl; e++)
		if (!d.gate[e] || !d.up[e] || !d.down[e])
			return fail(MOE_ERR_INVALID, "moe_layer_create: expert %lld has no weights",
				    (long long)e);
	if (kq && nl < d.n_experts)
		return fail(MOE_ERR_UNSUPPORTED, "moe_layer_create: K-quant experts on one GPU only");
	moe_layer *L = new moe_layer();
	L->d = d;
	L->qt_gu = qt_gu;
	L->qt_dn = qt_dn;
	L->mma_ok = !kq && moe::expert_mma_supported(d.qtype, (int)d.d_model) &&
		    moe::expert_mma_supported(d.qtype, (int)d.d_ff);
	for (int64_t e = first; e < first + nl; e++)
		L->mma_ok = L->mma_ok && ((uintptr_t)d.gate[e] % 16 == 0) &&
			    ((uintptr_t)d.up[e] % 16 == 0) && ((uintptr_t)d.down[e] % 16 == 0);
	L->d.first_expert = first;
	L->d.n_local = nl;
	L->d.gate = L->d.up = L->d.down = nullptr;
	std::vector<const void *> host(3 * d.n_experts);
	for (int64_t e = 0; e < d.n_experts; e++) {
		host[e] = d.gate[e];
		host[d.n_experts + e] = d.up[e];
		host[2 * d.n_experts + e] = d.down[e];
	}
	cudaError_t e = cudaMalloc(&L->dptrs, host.size() * sizeof(void *));
	if (e == cudaSuccess)
		e = cudaMemcpy(L->dptrs, host.data(), host.size() * sizeof(void *),
			       cudaMemcpyHostToDevice);
	const int qt = (int)d.qtype, D = (int)d.d_model, F = (int)d.d_ff;
	L->gemm_ok = !kq && L->mma_ok && moe::expert_gemm_supported(qt, F, D, 1) &&
		     moe::expert_gemm_supported(qt, D, F, 0);
	if (e == cudaSuccess && L->gemm_ok) {
		// tensor maps of every local expert matrix for the prefill GEMM
		const size_t mb = moe::weight_map_bytes();
		std::vector<uint8_t> maps(3 * d.n_experts * mb, 0);
		for (int64_t x = first; x < first + nl && L->gemm_ok; x++)
			L->gemm_ok = moe::encode_weight_map(&maps[x * mb], host[x], qt, F, D) &&
				     moe::encode_weight_map(&maps[(d.n_experts + x) * mb],
							    host[d.n_experts + x], qt, F, D) &&
				     moe::encode_weight_map(&maps[(2 * d.n_experts + x) * mb],
							    host[2 * d.n_experts + x], qt, D, F);
		if (L->gemm_ok) {
			e = cudaMalloc(&L->wmaps, maps.size());
			if (e == cudaSuccess)
				e = cudaMemcpy(L->wmaps, maps.data(), maps.size(), cudaMemcpyHostToDevice);
		}
	}
	if (e == cudaSuccess && nl < d.n_experts) {
		// rows of every (token, slot) pair of a decode batch, twice; the
		// counters; every rank's ids and tokens (token-sharded)
		L->y_half = (int64_t)moe::decode_max_t() * d.top_k * d.d_model;
		L->xl = moe::ep_layout(L->y_half, d.d_model);
		e = cudaMalloc(&L->xbuf, L->xl.bytes);
		if (e == cudaSuccess)
			e = cudaMemset(L->xbuf, 0, L->xl.bytes);
		if (e == cudaSuccess)
			e = cudaDeviceSynchronize();
	}
	if (e != cudaSuccess) {
		cudaFree(L->dptrs);
		cudaFree(L->wmaps);
		cudaFree(L->xbuf);
		delete L;
		return cuda_fail(e, "moe_layer_create");
	}
	*out = L;
	return MOE_OK;
}

int moe_layer_destroy(moe_layer *L)
{
	if (!L)
		return MOE_OK;
	if (g.init)
		cudaStreamSynchronize(g.stream);
	cudaFree(L->dptrs);
	cudaFree(L->wmaps);
	cudaFree(L->scratch);
	for (void *p : L->opened)
		cudaIpcCloseMemHandle(p);
	cudaFree(L->d_ybuf);
	cudaFree(L->d_inbound);
	cudaFree(L->d_routed);
	cudaFree(L->d_xg);
	cudaFree(L->d_idg);
	cudaFree(L->xbuf);
	cudaFree(L->a2a.buf);
	cudaFree(L->a2a.meta);
	if (L->a2a.host)
		cudaFreeHost(L->a2a.host);
	for (auto &set : L->prof)
		for (auto ev : set)
			cudaEventDestroy(ev);
	delete L;
	return MOE_OK;
}

int moe_layer_forward(moe_layer *L, const float *x, float *out, int64_t T, int flags,
		      void *stream)
{
	if (!L)
		return fail(MOE_ERR_INVALID, "moe_layer_forward: null layer");
	if (T < 0 || T > (1 << 22))
		return fail(MOE_ERR_INVALID, "moe_layer_forward: T = %lld", (long long)T);
	L->lastT = T;
	if (T == 0)
		return MOE_OK;
	if (!x || !out)
		return fail(MOE_ERR_INVALID, "moe_layer_forward: null x/out");
	if (int rc = layer_scratch(L, T))
		return rc;
	const moe_layer_desc &d = L->d;
	flags |= d.flags;
	cudaStream_t st = stream ? (cudaStream_t)stream : g.stream;
	const int NE = (int)d.n_experts, K = (int)d.top_k, D = (int)d.d_model, F = (int)d.d_ff;
	const int lanes = (flags & MOE_LANES_AVX2) ? 8 : 16;
	const bool prof = (flags & MOE_PROFILE) != 0;
	cudaEvent_t *ev = nullptr;
	// inside a stream capture an event record must be "external" to record a
	// timestamp each time the graph runs
	cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
	CK(cudaStreamIsCapturing(st, &cap));
	auto record = [&](cudaEvent_t e) {
		return cap == cudaStreamCaptureStatusActive
			       ? cudaEventRecordWithFlags(e, st, cudaEventRecordExternal)
			       : cudaEventRecord(e, st);
	};
	const bool simple = (flags & MOE_SIMPLE) || !L->mma_ok;
	const int q4 = d.qtype == MOE_Q4_0;
	const int mode_exact = (flags & MOE_TOPK_EXACT) ? 1 : 0, renorm = (flags & MOE_RENORM) ? 1 : 0;

	// decode-sized batch on one GPU: the whole layer in one fused kernel
	const bool ep_ready = L->ep_world > 1 && L->d_ybuf;
	// token-sharded expert parallelism: this rank's own tokens
	const bool shard = (flags & MOE_EP_SHARDED) && d.n_local < d.n_experts;
	if (shard && !ep_ready && !nccl.comm)
		return fail(MOE_ERR_INVALID, "moe_layer_forward: MOE_EP_SHARDED needs the ranks "
			    "connected (moe_layer_set_peers and/or moe_ep_init)");
	if (ktype(L->qt_gu)) {
		// K-quant experts (kquant.cu): router, routing, tokens to Q8_K, the
		// gate/up and down GEMVs, combine
		L->last_pairs = T * K;
		if (moe::router_tiled_ok(D, NE))
			CK(moe::launch_router_tiled(x, d.router_w, (int)T, D, NE, lanes, L->logits, nullptr,
						    0, st));
		else
			CK(moe::launch_router_logits(x, d.router_w, (int)T, D, NE, lanes, L->logits, st));
		if (T <= 256 && moe::route_small_smem((int)T, NE, K) <= 160 * 1024) {
			CK(moe::launch_route_small(L->logits, d.router_bias, (int)T, NE, K, lanes, mode_exact,
						   renorm, 0, NE, L->ids, L->wts, L->counts, L->offsets,
						   L->perm, L->pos_of, L->active, L->n_active, L->err, L->work,
						   st));
		} else {
			CK(moe::launch_router_topk(L->logits, d.router_bias, (int)T, NE, K, lanes,
						   mode_exact, renorm, L->ids, L->wts, nullptr, st));
			CK(moe::launch_dispatch(L->ids, (int)(T * K), NE, 0, NE, L->counts, L->offsets,
						L->perm, L->pos_of, L->active, L->n_active, L->err, L->work,
						st));
		}
		CK(moe::launch_quantize_q8k(x, (int)T, D, L->q8k, st));
		moe::KqArgs ka{};
		ka.w1 = L->dptrs;
		ka.w2 = L->dptrs + NE;
		ka.rows = F;
		ka.cols = D;
		ka.K = K;
		ka.first_expert = 0;
		ka.n_local = NE;
		ka.counts = L->counts;
		ka.offsets = L->offsets;
		ka.perm = L->perm;
		ka.x8 = L->q8k;
		ka.h = L->h;
		CK(moe::launch_kq_gate_up(ka, L->qt_gu, st));
		moe::KqArgs kd = ka;
		kd.w1 = L->dptrs + 2 * NE;
		kd.w2 = nullptr;
		kd.rows = D;
		kd.cols = F;
		kd.hin = L->h;
		kd.out = L->Y;
		CK(moe::launch_kq_down(kd, L->qt_dn, st));
		CK(moe::launch_combine(L->Y, L->wts, (int)T, K, D, out, st));
		return MOE_OK;
	}
	const int64_t world_pairs = shard ? (int64_t)L->ep_world * T * K : T * K;
	// one token on one GPU: its K experts through the single-row GEMV
	// (gemv.cu), when that is the faster kernel for the expert type
	const bool t1 = T == 1 && !simple && ((flags & MOE_FORCE_T1) || t1_on(d.qtype)) &&
			!(flags & (MOE_NO_FUSE | MOE_FORCE_GEMM | MOE_NO_T1)) &&
			d.n_local == d.n_experts && !ep_ready && !shard && (uintptr_t)x % 16 == 0 &&
			(uintptr_t)d.router_w % 16 == 0 && moe::router_t1_ok(D, NE, K) &&
			moe::expert_t1_chunks(d.qtype, D, F, K) > 0;
	if (!simple && !t1 && !(flags & (MOE_NO_FUSE | MOE_FORCE_GEMM)) && (d.n_local == d.n_experts || ep_ready) &&
	    moe::decode_supported(d.qtype, T, D, F, NE, K, world_pairs, (uintptr_t)x,
				  (uintptr_t)d.router_w, (uintptr_t)out)) {
		uint64_t *stamps = nullptr;
		if (prof && L->prof_used < kStampRecords) {
			stamps = L->stamps + L->prof_used * moe::sm_count() * moe::decode_stamps();
			if (L->prof_fused.size() <= L->prof_used)
				L->prof_fused.resize(L->prof_used + 1);
			L->prof_fused[L->prof_used++] = 1;
		}
		moe::DecodeArgs a{};
		a.x = x;
		a.router_w = d.router_w;
		a.router_bias = d.router_bias;
		a.dptrs = L->dptrs;
		a.T = (int)T;
		a.D = D;
		a.F = F;
		a.NE = NE;
		a.K = K;
		a.mode_exact = mode_exact;
		a.renorm = renorm;
		a.logits = L->logits;
		a.x16 = L->x16;
		a.h16 = L->h16;
		a.Y = L->Y;
		a.out = out;
		a.ids = L->ids;
		a.wts = L->wts;
		a.counts = L->counts;
		a.offsets = L->offsets;
		a.perm = L->perm;
		a.active = L->active;
		a.n_active = L->n_active;
		a.err = L->err;
		a.gbar = L->gbar;
		a.stamps = stamps;
		a.first_expert = (int)d.first_expert;
		a.n_local = (int)d.n_local;
		a.rank = L->ep_rank;
		a.world = ep_ready ? L->ep_world : 1;
		a.shard = shard ? 1 : 0;
		a.ybuf = L->d_ybuf;
		a.ybuf_half = L->y_half;
		a.inbound = L->d_inbound;
		a.routed = L->d_routed;
		a.xg = L->d_xg;
		a.idg = L->d_idg;
		a.launches = ep_ready ? reinterpret_cast<unsigned long long *>(L->xbuf + L->xl.launches)
				      : nullptr;
		a.shard_launches = ep_ready ? reinterpret_cast<unsigned long long *>(
						      L->xbuf + L->xl.shard_launches)
					    : nullptr;
		a.ep_wait_ns = L->ep_wait_ns;
		CK(moe::launch_decode_layer(a, d.qtype, lanes, st));
		L->last_pairs = world_pairs;
		return MOE_OK;
	}

	if (prof) {
		while (L->prof.size() <= L->prof_used) {
			std::array<cudaEvent_t, 6> set{};
			for (auto &e : set)
				CK(cudaEventCreate(&e));
			L->prof.push_back(set);
		}
		if (L->prof_fused.size() <= L->prof_used)
			L->prof_fused.resize(L->prof_used + 1);
		L->prof_fused[L->prof_used] = 0;
		ev = L->prof[L->prof_used++].data();
		CK(record(ev[0]));
	}
	if (shard)
		return forward_sharded_a2a(L, x, out, T, flags, st, ev);
	L->last_pairs = T * K;
	if (t1) {
		// [0] + [1] router, top-k and dispatch in one launch; gate/up rows
		// of the K experts -> L->h ([2K][F]); down in column chunks -> L->Y
		// ([chunks][K][D]); combine
		CK(moe::launch_router_t1(x, d.router_w, d.router_bias, D, NE, K, lanes, mode_exact,
					 renorm, L->logits, L->ids, L->wts, L->counts, L->offsets,
					 L->perm, L->pos_of, L->active, L->n_active, L->err, L->work,
					 L->t1cnt, st));
		if (prof) {
			CK(record(ev[1]));
			CK(record(ev[2]));
		}
		for (int stage = 0; stage < 3; stage++) {
			CK(moe::launch_expert_t1(stage, L->dptrs, L->ids, L->wts, d.qtype, D, F, NE, K, x,
						 L->h, L->Y, out, L->err, st));
			if (prof)
				CK(record(ev[3 + stage]));
		}
		return MOE_OK;
	}
	// prefill-sized batches: grouped GEMMs on tcgen05 (the tokens are gathered
	// into pair order after the dispatch instead of split in token order)
	const bool gemm = !simple && L->gemm_ok && !(flags & MOE_FORCE_GEMV) &&
			  (T > moe::decode_max_t() || (flags & MOE_FORCE_GEMM)) && (uintptr_t)x % 16 == 0;
	// [0] router logits (+ the fp16 split of x the MMA kernels read)
	if (moe::router_tiled_ok(D, NE)) {
		CK(moe::launch_router_tiled(x, d.router_w, (int)T, D, NE, lanes, L->logits,
					    (simple || gemm) ? nullptr : L->x16, q4, st));
	} else {
		CK(moe::launch_router_logits(x, d.router_w, (int)T, D, NE, lanes, L->logits, st));
		if (!simple && !gemm)
			CK(moe::launch_split_f16(x, T, D, d.qtype, L->x16, st));
	}
	if (prof)
		CK(record(ev[1]));
	// [1] softmax + top-k + dispatch
	if (T <= 256 && moe::route_small_smem((int)T, NE, K) <= 160 * 1024) {
		CK(moe::launch_route_small(L->logits, d.router_bias, (int)T, NE, K, lanes, mode_exact,
					   renorm, (int)d.first_expert, (int)d.n_local, L->ids, L->wts,
					   L->counts, L->offsets, L->perm, L->pos_of, L->active,
					   L->n_active, L->err, L->work, st));
	} else {
		CK(moe::launch_router_topk(L->logits, d.router_bias, (int)T, NE, K, lanes, mode_exact,
					   renorm, L->ids, L->wts, nullptr, st));
		CK(moe::launch_dispatch(L->ids, (int)(T * K), NE, (int)d.first_expert,
					(int)d.n_local, L->counts, L->offsets, L->perm, L->pos_of,
					L->active, L->n_active, L->err, L->work, st));
	}
	if (d.n_local < d.n_experts)
		CK(cudaMemsetAsync(L->Y, 0, (size_t)T * K * D * sizeof(float), st));

	const void *const *dp = L->dptrs;
	if (prof)
		CK(record(ev[2]));
	if (gemm) {
		const int64_t pairs = T * K;
		CK(moe::launch_gather_split(x, L->perm, pairs, D, K, L->x16p, st));
		const size_t mb = moe::weight_map_bytes();
		moe::GemmArgs gu{};
		gu.maps1 = L->wmaps;
		gu.maps2 = (const uint8_t *)L->wmaps + NE * mb;
		gu.qtype = d.qtype;
		gu.rows = F;
		gu.cols = D;
		gu.n_local = (int)d.n_local;
		gu.counts = L->counts;
		gu.offsets = L->offsets;
		gu.perm = L->perm;
		gu.active = L->active;
		gu.n_active = L->n_active;
		gu.out_perm = 0;
		gu.in16 = L->x16p;
		gu.out16 = L->h16;
		gu.dual = 1;
		gu.err = L->err;
		CK(moe::launch_expert_gemm(gu, pairs, st));
		if (prof)
			CK(record(ev[3]));
		moe::GemmArgs dn = gu;
		dn.maps1 = (const uint8_t *)L->wmaps + 2 * NE * mb;
		dn.maps2 = nullptr;
		dn.rows = D;
		dn.cols = F;
		dn.out_perm = 1;
		dn.in16 = L->h16;
		dn.out16 = nullptr;
		dn.out = L->Y;
		dn.dual = 0;
		CK(moe::launch_expert_gemm(dn, pairs, st));
	} else if (simple) {
		moe::GemvArgs gu{};
		gu.w1 = dp;
		gu.w2 = dp + NE;
		gu.qtype = d.qtype;
		gu.rows = F;
		gu.cols = D;
		gu.NE = NE;
		gu.K = K;
		gu.first_expert = (int)d.first_expert;
		gu.n_local = (int)d.n_local;
		gu.counts = L->counts;
		gu.offsets = L->offsets;
		gu.perm = L->perm;
		gu.in_perm = 1;
		gu.out_perm = 0;
		gu.in = x;
		gu.out = L->h;
		gu.dual = 1;
		CK(moe::launch_expert_gemv(gu, st));
		if (prof)
			CK(record(ev[3]));
		moe::GemvArgs dn = gu;
		dn.w1 = dp + 2 * NE;
		dn.w2 = nullptr;
		dn.rows = D;
		dn.cols = F;
		dn.in_perm = 0;
		dn.out_perm = 1;
		dn.in = L->h;
		dn.out = L->Y;
		dn.dual = 0;
		CK(moe::launch_expert_gemv(dn, st));
	} else {
		moe::MmaArgs gu{};
		gu.w1 = dp;
		gu.w2 = dp + NE;
		gu.qtype = d.qtype;
		gu.rows = F;
		gu.cols = D;
		gu.NE = NE;
		gu.K = K;
		gu.first_expert = (int)d.first_expert;
		gu.n_local = (int)d.n_local;
		gu.counts = L->counts;
		gu.offsets = L->offsets;
		gu.perm = L->perm;
		gu.in_perm = 1;
		gu.out_perm = 0;
		gu.in16 = L->x16;
		gu.out16 = L->h16;
		gu.dual = 1;
		gu.err = L->err;
		gu.active = L->active;
		gu.n_active = L->n_active;
		gu.work = L->work;
		CK(moe::launch_expert_mma(gu, st));
		if (prof)
			CK(record(ev[3]));
		moe::MmaArgs dn = gu;
		dn.w1 = dp + 2 * NE;
		dn.w2 = nullptr;
		dn.rows = D;
		dn.cols = F;
		dn.in_perm = 0;
		dn.out_perm = 1;
		dn.in16 = L->h16;
		dn.out16 = nullptr;
		dn.out = L->Y;
		dn.dual = 0;
		dn.work = L->work + 1;
		CK(moe::launch_expert_mma(dn, st));
	}
	if (prof)
		CK(record(ev[4]));

	CK(moe::launch_combine(L->Y, L->wts, (int)T, K, D, out, st));
	// expert parallelism outside the fused kernel: every rank holds the
	// combine of its own experts' rows; their sum is the layer output
	if (d.n_local < d.n_experts && nccl.comm)
		CK_NCCL(nccl.all_reduce(out, out, (size_t)T * D, ncclFloat32, ncclSum, nccl.comm, st));
	if (prof)
		CK(record(ev[5]));
	return MOE_OK;
}

int moe_layer_stage_ms(moe_layer *L, float *ms, int n)
{
	if (!L || !ms || n < 5)
		return fail(MOE_ERR_INVALID, "moe_layer_stage_ms: need a layer and 5 floats");
	if (L->prof_used == 0)
		return fail(MOE_ERR_INVALID, "moe_layer_stage_ms: no MOE_PROFILE forward to report");
	for (int i = 0; i < 5; i++)
		ms[i] = 0.0f;
	CK(cudaDeviceSynchronize());  // the forwards may have run on a caller stream
	const int grid = moe::sm_count(), ns = moe::decode_stamps();
	std::vector<uint64_t> st((size_t)grid * ns);
	for (size_t c = 0; c < L->prof_used; c++) {
		if (c < L->prof_fused.size() && L->prof_fused[c]) {
			// phase boundaries: latest CTA per boundary, from the earliest start
			CK(cudaMemcpy(st.data(), L->stamps + c * grid * ns, st.size() * 8,
				      cudaMemcpyDeviceToHost));
			int ends[5];
			moe::decode_stage_ends(ends);
			uint64_t bnd[6] = {UINT64_MAX, 0, 0, 0, 0, 0};
			for (int b = 0; b < grid; b++) {
				bnd[0] = std::min(bnd[0], st[(size_t)b * ns]);
				for (int i = 0; i < 5; i++)
					bnd[i + 1] = std::max(bnd[i + 1], st[(size_t)b * ns + ends[i]]);
			}
			for (int i = 0; i < 5; i++)
				ms[i] += (float)((double)(bnd[i + 1] - bnd[i]) * 1e-6);
			continue;
		}
		for (int i = 0; i < 5; i++) {
			float t = 0.0f;
			CK(cudaEventElapsedTime(&t, L->prof[c][i], L->prof[c][i + 1]));
			ms[i] += t;
		}
	}
	if (n >= 6)
		ms[5] = (float)L->prof_used;
	L->prof_used = 0;
	return MOE_OK;
}

int moe_layer_ipc_handle(moe_layer *L, void *handle)
{
	if (!L || !handle)
		return fail(MOE_ERR_INVALID, "moe_layer_ipc_handle: null argument");
	if (!L->xbuf)
		return fail(MOE_ERR_INVALID, "moe_layer_ipc_handle: the layer computes every expert "
			    "(no exchange buffer)");
	cudaIpcMemHandle_t h;
	CK(cudaIpcGetMemHandle(&h, L->xbuf));
	memcpy(handle, &h, sizeof(h));
	return MOE_OK;
}

int moe_layer_set_peers(moe_layer *L, int rank, int world, const void *handles)
{
	if (!L || !handles)
		return fail(MOE_ERR_INVALID, "moe_layer_set_peers: null argument");
	if (!L->xbuf)
		return fail(MOE_ERR_INVALID, "moe_layer_set_peers: the layer computes every expert");
	if (world < 2 || world > moe::kMaxEpRanks || rank < 0 || rank >= world)
		return fail(MOE_ERR_INVALID, "moe_layer_set_peers: rank %d of %d (2..%d ranks)", rank,
			    world, moe::kMaxEpRanks);
	if (L->d_ybuf)
		return fail(MOE_ERR_INVALID, "moe_layer_set_peers: peers already set");
	std::vector<float *> yb(world);
	std::vector<unsigned long long *> inb(world), rtd(world);
	std::vector<__half *> xg(world);
	std::vector<int32_t *> idg(world);
	const auto *hs = static_cast<const cudaIpcMemHandle_t *>(handles);
	for (int r = 0; r < world; r++) {
		void *base = L->xbuf;
		if (r != rank) {
			cudaError_t e = cudaIpcOpenMemHandle(&base, hs[r], cudaIpcMemLazyEnablePeerAccess);
			if (e != cudaSuccess) {
				for (void *p : L->opened)
					cudaIpcCloseMemHandle(p);
				L->opened.clear();
				return cuda_fail(e, "moe_layer_set_peers: cudaIpcOpenMemHandle");
			}
			L->opened.push_back(base);
		}
		char *cb = static_cast<char *>(base);
		yb[r] = reinterpret_cast<float *>(cb);
		inb[r] = reinterpret_cast<unsigned long long *>(cb + L->xl.inbound);
		rtd[r] = reinterpret_cast<unsigned long long *>(cb + L->xl.routed);
		idg[r] = reinterpret_cast<int32_t *>(cb + L->xl.idg);
		xg[r] = reinterpret_cast<__half *>(cb + L->xl.xg);
	}
	const size_t pb = world * sizeof(void *);
	CK(cudaMalloc(&L->d_ybuf, pb));
	CK(cudaMalloc(&L->d_inbound, pb));
	CK(cudaMalloc(&L->d_routed, pb));
	CK(cudaMalloc(&L->d_xg, pb));
	CK(cudaMalloc(&L->d_idg, pb));
	CK(cudaMemcpy(L->d_ybuf, yb.data(), pb, cudaMemcpyHostToDevice));
	CK(cudaMemcpy(L->d_inbound, inb.data(), pb, cudaMemcpyHostToDevice));
	CK(cudaMemcpy(L->d_routed, rtd.data(), pb, cudaMemcpyHostToDevice));
	CK(cudaMemcpy(L->d_xg, xg.data(), pb, cudaMemcpyHostToDevice));
	CK(cudaMemcpy(L->d_idg, idg.data(), pb, cudaMemcpyHostToDevice));
	L->ep_rank = rank;
	L->ep_world = world;
	return MOE_OK;
}

int moe_layer_phase_stamps(moe_layer *L, uint64_t *out, int n)
{
	if (!L || !out)
		return fail(MOE_ERR_INVALID, "moe_layer_phase_stamps: null argument");
	const int grid = moe::sm_count(), ns = moe::decode_stamps();
	size_t rec = SIZE_MAX;
	for (size_t c = 0; c < L->prof_used && c < L->prof_fused.size(); c++)
		if (L->prof_fused[c])
			rec = c;
	if (rec == SIZE_MAX)
		return fail(MOE_ERR_INVALID, "moe_layer_phase_stamps: no profiled fused forward");
	if (n < grid * ns)
		return fail(MOE_ERR_INVALID, "moe_layer_phase_stamps: need %d values", grid * ns);
	CK(cudaDeviceSynchronize());
	CK(cudaMemcpy(out, L->stamps + rec * grid * ns, (size_t)grid * ns * 8,
		      cudaMemcpyDeviceToHost));
	return grid * ns;
}

int moe_layer_routing(moe_layer *L, int32_t *ids, float *weights, int32_t *counts,
		      int32_t *offsets, int32_t *perm)
{
	if (!L)
		return fail(MOE_ERR_INVALID, "moe_layer_routing: null layer");
	const int64_t T = L->lastT, K = L->d.top_k, NE = L->d.n_experts;
	if (int rc = moe_layer_status(L))
		return rc;
	if (T == 0)
		return MOE_OK;
	if (ids)
		CK(cudaMemcpy(ids, L->ids, T * K * 4, cudaMemcpyDeviceToHost));
	if (weights)
		CK(cudaMemcpy(weights, L->wts, T * K * 4, cudaMemcpyDeviceToHost));
	if (counts)
		CK(cudaMemcpy(counts, L->counts, NE * 4, cudaMemcpyDeviceToHost));
	if (offsets)
		CK(cudaMemcpy(offsets, L->offsets, (NE + 1) * 4, cudaMemcpyDeviceToHost));
	if (perm)
		CK(cudaMemcpy(perm, L->perm, L->last_pairs * 4, cudaMemcpyDeviceToHost));
	return MOE_OK;
}

int moe_layer_status(moe_layer *L)
{
	if (!L)
		return fail(MOE_ERR_INVALID, "moe_layer_status: null layer");
	if (!L->err)
		return MOE_OK;  // no forward has run
	CK(cudaDeviceSynchronize());  // the forward may have run on a caller stream
	int32_t err = 0;
	CK(cudaMemcpy(&err, L->err, 4, cudaMemcpyDeviceToHost));
	return take_error(L, err);
}

int moe_layer_set_wait_ms(moe_layer *L, int ms)
{
	if (!L || ms <= 0)
		return fail(MOE_ERR_INVALID, "moe_layer_set_wait_ms: need a layer and ms > 0");
	L->ep_wait_ns = (uint64_t)ms * 1000000ull;
	return MOE_OK;
}

int moe_layer_ep_reset(moe_layer *L)
{
	if (!L)
		return fail(MOE_ERR_INVALID, "moe_layer_ep_reset: null layer");
	CK(cudaDeviceSynchronize());
	if (L->xbuf)
		CK(cudaMemset(L->xbuf + L->xl.inbound, 0, L->xl.idg - L->xl.inbound));
	if (L->err) {
		CK(cudaMemset(L->err, 0, 4));
		CK(cudaMemset(L->gbar, 0, moe::decode_barrier_bytes(moe::sm_count())));
	}
	CK(cudaDeviceSynchronize());
	return MOE_OK;
}

// ---------------------------------------------------------------- dense GEMV
}  // extern "C"

namespace moe {
// The dense projection behind moe_gemv_device and the model forward: one
// "expert" holding all m rows of x (counts = {m}, offsets = {0, m}).  The
// metadata (and the GEMM's weight tensor map) and the fp16 split of x live
// in the caller's scratch, so calls sharing one scratch must be ordered on
// one stream.  m == 1 with a supported shape takes the single-row GEMV,
// which needs no scratch and issues no copy (graph-capturable).
struct DenseMeta {
	alignas(64) uint8_t map[128];  // prefill GEMM: the weight matrix's tensor map
	const void *w;
	int32_t counts[1], offsets[2], err[1], active[1], n_active[1], work[1];
};

void dense_scratch_free(DenseScratch &s)
{
	if (s.meta)
		cudaFree(s.meta);
	if (s.x16)
		cudaFree(s.x16);
	s = DenseScratch{};
}

int dense_forward(DenseScratch &s, const void *w, int qtype, int64_t rows, int64_t cols,
		  const float *x, int64_t m, float *y, int32_t *err, cudaStream_t st)
{
	if ((qtype != MOE_Q8_0 && qtype != MOE_Q4_0) || cols % QK || rows <= 0 || m < 0)
		return fail(MOE_ERR_INVALID, "dense projection: qtype %d rows %lld cols %lld", qtype,
			    (long long)rows, (long long)cols);
	if (m == 0)
		return MOE_OK;
	// one activation row (decode): the memory-bound GEMV, no scratch
	if (m == 1 && moe::gemv1_supported(qtype, rows, cols, (uintptr_t)w, (uintptr_t)x, (uintptr_t)y)) {
		CK(moe::launch_gemv1(w, qtype, rows, cols, x, y, err, st));
		return MOE_OK;
	}
	using Meta = DenseMeta;
	if (!s.meta)
		CK(cudaMalloc(&s.meta, sizeof(Meta)));
	Meta *dmeta = static_cast<Meta *>(s.meta);
	auto ensure_x16 = [&](size_t need) -> int {
		if (need <= s.x16_bytes)
			return MOE_OK;
		CK(cudaStreamSynchronize(st));
		if (s.x16)
			cudaFree(s.x16);
		s.x16 = nullptr;
		s.x16_bytes = 0;
		CK(cudaMalloc(&s.x16, need));
		s.x16_bytes = need;
		return MOE_OK;
	};
	__half *&x16 = s.x16;
	Meta h{};
	h.w = w;
	h.counts[0] = (int32_t)m;
	h.offsets[1] = (int32_t)m;
	h.n_active[0] = 1;
	// prefill-sized batches (dense projections, lm_head): the tcgen05 GEMM
	// of the expert layers with one expert; its weight tensor map views the
	// GGUF rows where they are
	if (m > moe::decode_max_t() && m <= INT32_MAX / 2 &&
	    moe::expert_gemm_supported(qtype, (int)rows, (int)cols, 0) && (uintptr_t)w % 16 == 0 &&
	    (uintptr_t)x % 16 == 0 && (uintptr_t)y % 16 == 0 &&
	    moe::encode_weight_map(h.map, w, qtype, (int)rows, (int)cols)) {
		CK(cudaMemcpyAsync(dmeta, &h, sizeof(Meta), cudaMemcpyHostToDevice, st));
		if (int rc = ensure_x16((size_t)m * 2 * cols * sizeof(__half)))
			return rc;
		CK(moe::launch_gather_split(x, nullptr, m, (int)cols, 1, x16, st));
		moe::GemmArgs a{};
		a.maps1 = dmeta->map;
		a.qtype = qtype;
		a.rows = (int)rows;
		a.cols = (int)cols;
		a.n_local = 1;
		a.counts = dmeta->counts;
		a.offsets = dmeta->offsets;
		a.perm = nullptr;
		a.active = dmeta->active;
		a.n_active = dmeta->n_active;
		a.out_perm = 0;
		a.in16 = x16;
		a.out = y;
		a.dual = 0;
		a.err = err;
		CK(moe::launch_expert_gemm(a, m, st));
		return MOE_OK;
	}
	CK(cudaMemcpyAsync(dmeta, &h, sizeof(Meta), cudaMemcpyHostToDevice, st));
	const bool mma = moe::expert_mma_supported(qtype, (int)cols) && (uintptr_t)w % 16 == 0;
	if (mma) {
		if (int rc = ensure_x16((size_t)m * 2 * cols * sizeof(__half)))
			return rc;
		CK(moe::launch_split_f16(x, m, (int)cols, qtype, x16, st));
		moe::MmaArgs a{};
		a.w1 = reinterpret_cast<const void *const *>(&dmeta->w);
		a.qtype = qtype;
		a.rows = (int)rows;
		a.cols = (int)cols;
		a.NE = 1;
		a.K = 1;
		a.first_expert = 0;
		a.n_local = 1;
		a.counts = dmeta->counts;
		a.offsets = dmeta->offsets;
		a.perm = nullptr;
		a.in_perm = a.out_perm = 0;
		a.in16 = x16;
		a.out = y;
		a.dual = 0;
		a.err = err;
		a.active = dmeta->active;
		a.n_active = dmeta->n_active;
		a.work = dmeta->work;
		CK(moe::launch_expert_mma(a, st));
		return MOE_OK;
	}
	moe::GemvArgs a{};
	a.w1 = reinterpret_cast<const void *const *>(&dmeta->w);
	a.qtype = qtype;
	a.rows = (int)rows;
	a.cols = (int)cols;
	a.NE = 1;
	a.K = 1;
	a.first_expert = 0;
	a.n_local = 1;
	a.counts = dmeta->counts;
	a.offsets = dmeta->offsets;
	a.perm = nullptr;
	a.in_perm = a.out_perm = 0;
	a.in = x;
	a.out = y;
	a.dual = 0;
	CK(moe::launch_expert_gemv(a, st));
	return MOE_OK;
}
}  // namespace moe

extern "C" {

int moe_gemv_device(const void *w, int qtype, int64_t rows, int64_t cols, const float *x,
		    int64_t m, float *y, void *stream)
{
	if (int rc = ensure_init())
		return rc;
	if ((qtype != MOE_Q8_0 && qtype != MOE_Q4_0) || cols % QK || rows <= 0 || m < 0)
		return fail(MOE_ERR_INVALID, "moe_gemv_device: qtype %d rows %lld cols %lld", qtype,
			    (long long)rows, (long long)cols);
	if (m == 0)
		return MOE_OK;
	cudaStream_t st = stream ? (cudaStream_t)stream : g.stream;
	if (!g.gemv_err) {
		CK(cudaMalloc(&g.gemv_err, 4));
		CK(cudaMemset(g.gemv_err, 0, 4));
	}
	// every path's bounded waits report to the library's GEMV error word
	// (moe_sync); the scratch is per calling thread
	static thread_local moe::DenseScratch scratch;
	return moe::dense_forward(scratch, w, qtype, rows, cols, x, m, y, g.gemv_err, st);
}

// ---------------------------------------------------------------- drop-ins
int moe_tensor_mma_transposed_2x2_status(moe_tensor_t *ret, const moe_tensor_t *lhs,
					 const moe_tensor_t *rhs, const moe_tensor_t *add)
{
	if (!ret || !lhs || !rhs)
		return fail(MOE_ERR_INVALID, "tensor_mma_transposed_2x2: null tensor");
	if (lhs->ndim != 2 || rhs->ndim != 2 || lhs->dim[1] != rhs->dim[1] ||
	    lhs->type != MOE_F32 || !lhs->data || !ret->data)
		return fail(MOE_ERR_INVALID, "tensor_mma_transposed_2x2: shape/type mismatch "
			    "(matmul.c:277-279 asserts)");
	if (rhs->type != MOE_F32 && rhs->type != MOE_Q8_0 && rhs->type != MOE_Q4_0)
		return fail(MOE_ERR_UNSUPPORTED, "tensor_mma_transposed_2x2: rhs dtype %d",
			    rhs->type);
	const int64_t m = (int64_t)lhs->dim[0], k = (int64_t)lhs->dim[1], n = (int64_t)rhs->dim[0];
	if (ret->maxcap < (uint64_t)(m * n))
		return fail(MOE_ERR_INVALID, "tensor_mma_transposed_2x2: ret maxcap %llu < %lld",
			    (unsigned long long)ret->maxcap, (long long)(m * n));
	if (add && add->totlen != (uint64_t)(m * n) && add->totlen != (uint64_t)n)
		return fail(MOE_ERR_INVALID, "tensor_mma_transposed_2x2: add length %llu",
			    (unsigned long long)add->totlen);
	if (rhs->type != MOE_F32 && k % QK)
		return fail(MOE_ERR_INVALID, "tensor_mma_transposed_2x2: k %% 32 != 0");
	if (int rc = ensure_init())
		return rc;
	const void *dw;
	if (int rc = resolve(tensor_host_ptr(rhs), tensor_bytes(rhs), &dw))
		return rc;
	// mma_init (matmul.c:13-33) reshapes ret to [m, n]
	ret->ndim = 2;
	ret->dim[0] = (uint64_t)m;
	ret->dim[1] = (uint64_t)n;
	ret->totlen = (uint64_t)(m * n);
	if (m == 0 || n == 0)
		return MOE_OK;
	const size_t xin = align_up(m * k * 4, 256), yout = align_up(m * n * 4, 256);
	const size_t addb = add ? align_up(add->totlen * 4, 256) : 0;
	if (int rc = ensure_dev_io(xin + yout + addb))
		return rc;
	if (int rc = ensure_pinned(std::max(m * k * 4, m * n * 4)))
		return rc;
	char *db = static_cast<char *>(g.dev_io);
	float *dx = (float *)db, *dy = (float *)(db + xin), *dadd = (float *)(db + xin + yout);
	CK(cudaMemcpyAsync(dx, lhs->data, m * k * 4, cudaMemcpyHostToDevice, g.stream));
	if (add)
		CK(cudaMemcpyAsync(dadd, add->data, add->totlen * 4, cudaMemcpyHostToDevice,
				   g.stream));
	if (rhs->type == MOE_F32) {
		// fp32 rhs: the exact lane-chain kernel of the router (matmul.c:169-245)
		CK(moe::launch_router_logits(dx, (const float *)dw, (int)m, (int)k, (int)n, 16, dy,
					     g.stream));
	} else {
		if (int rc = moe_gemv_device(dw, rhs->type, n, k, dx, m, dy, g.stream))
			return rc;
	}
	if (add)
		CK(moe::launch_add_bias(dy, dadd, m * n, (int64_t)add->totlen, g.stream));
	CK(cudaMemcpyAsync(g.pin, dy, m * n * 4, cudaMemcpyDeviceToHost, g.stream));
	CK(cudaStreamSynchronize(g.stream));
	if (int rc = take_gemv_error())
		return rc;
	memcpy(ret->data, g.pin, m * n * 4);
	return MOE_OK;
}

void moe_tensor_mma_transposed_2x2(moe_tensor_t *ret, const moe_tensor_t *lhs,
				   const moe_tensor_t *rhs, const moe_tensor_t *add)
{
	int rc = moe_tensor_mma_transposed_2x2_status(ret, lhs, rhs, add);
	if (rc) {
		fprintf(stderr, "moe_tensor_mma_transposed_2x2: %s\n", g_err.c_str());
		abort();
	}
}

int moe_fused_ffn_silu(const moe_tensor_t *in, moe_tensor_t *out, moe_tensor_t *gate,
		       const moe_tensor_t *gate_w, moe_tensor_t *up, const moe_tensor_t *up_w,
		       const moe_tensor_t *down_w)
{
	(void)up;
	// nn.c:503-507: applicable only to one token with quantized weights
	if (in->dim[0] != 1)
		return 0;
	if (gate_w->type == MOE_F32 || up_w->type == MOE_F32 || down_w->type == MOE_F32)
		return 0;
	auto die = [](const char *msg) {
		fprintf(stderr, "moe_fused_ffn_silu: %s\n", msg);
		abort();
	};
	if (gate_w->type != up_w->type || gate_w->type != down_w->type ||
	    (gate_w->type != MOE_Q8_0 && gate_w->type != MOE_Q4_0))
		die("unsupported weight types (Q8_0/Q4_0, all equal)");
	const int64_t k = (int64_t)in->dim[1];
	const int64_t inter = (int64_t)gate_w->dim[0];
	const int64_t out_n = (int64_t)down_w->dim[0];
	if (gate_w->dim[1] != (uint64_t)k || up_w->dim[0] != (uint64_t)inter ||
	    down_w->dim[1] != (uint64_t)inter || k % QK || inter % QK)
		die("shape mismatch");
	if (ensure_init())
		die(g_err.c_str());
	const void *dg, *du, *dd;
	if (resolve(gate_w->qdata, tensor_bytes(gate_w), &dg) ||
	    resolve(up_w->qdata, tensor_bytes(up_w), &du) ||
	    resolve(down_w->qdata, tensor_bytes(down_w), &dd))
		die(g_err.c_str());
	// a one-token, one-expert layer: counts {1}, offsets {0,1}, perm {0}
	struct Meta {
		const void *w[3];
		int32_t counts[1], offsets[2], perm[1];
	};
	const size_t xin = align_up(k * 4, 256), hb = align_up(inter * 4, 256);
	const size_t yb = align_up(out_n * 4, 256), mb = align_up(sizeof(Meta), 256);
	if (ensure_dev_io(xin + hb + yb + mb) || ensure_pinned(std::max(out_n, inter) * 4))
		die(g_err.c_str());
	char *db = static_cast<char *>(g.dev_io);
	float *dx = (float *)db, *dh = (float *)(db + xin), *dy = (float *)(db + xin + hb);
	Meta *dm = (Meta *)(db + xin + hb + yb);
	Meta hm{{dg, du, dd}, {1}, {0, 1}, {0}};
	if (cudaMemcpyAsync(dm, &hm, sizeof(Meta), cudaMemcpyHostToDevice, g.stream) ||
	    cudaMemcpyAsync(dx, in->data, k * 4, cudaMemcpyHostToDevice, g.stream))
		die("copy in failed");
	moe::GemvArgs a{};
	a.w1 = reinterpret_cast<const void *const *>(&dm->w[0]);
	a.w2 = reinterpret_cast<const void *const *>(&dm->w[1]);
	a.qtype = gate_w->type;
	a.rows = (int)inter;
	a.cols = (int)k;
	a.NE = 1;
	a.K = 1;
	a.first_expert = 0;
	a.n_local = 1;
	a.counts = dm->counts;
	a.offsets = dm->offsets;
	a.perm = dm->perm;
	a.in_perm = 0;
	a.out_perm = 0;
	a.in = dx;
	a.out = dh;
	a.dual = 1;
	if (moe::launch_expert_gemv(a, g.stream) != cudaSuccess)
		die("gate/up launch failed");
	moe::GemvArgs b = a;
	b.w1 = reinterpret_cast<const void *const *>(&dm->w[2]);
	b.w2 = nullptr;
	b.rows = (int)out_n;
	b.cols = (int)inter;
	b.in = dh;
	b.out = dy;
	b.dual = 0;
	if (moe::launch_expert_gemv(b, g.stream) != cudaSuccess)
		die("down launch failed");
	if (cudaMemcpyAsync(g.pin, dy, out_n * 4, cudaMemcpyDeviceToHost, g.stream) ||
	    cudaStreamSynchronize(g.stream))
		die("device error");
	memcpy(out->data, g.pin, out_n * 4);
	if (gate && gate->data) {
		if (cudaMemcpy(g.pin, dh, inter * 4, cudaMemcpyDeviceToHost))
			die("device error");
		memcpy(gate->data, g.pin, inter * 4);
	}
	return 1;
}

}  // extern "C"

// ---------------------------------------------------------------- layer drop-ins
namespace {

// the tensors of a drop-in forward against the experts' shape: input
// [T, Dw] fp32, router [NE, Dw] fp32, output room for T x Dw (host IO)
int check_io(const moe_tensor_t *input, const moe_tensor_t *output, const moe_tensor_t *gate_inp,
	     int64_t NE, int64_t Dw, int flags)
{
	if (!input || !output || !gate_inp)
		return fail(MOE_ERR_INVALID, "moe_ffn_forward: null tensor");
	if (input->type != MOE_F32 || gate_inp->type != MOE_F32 || input->ndim != 2 ||
	    gate_inp->ndim != 2)
		return fail(MOE_ERR_INVALID, "moe_ffn_forward: input/router must be 2-D fp32");
	const int64_t T = (int64_t)input->dim[0], D = (int64_t)input->dim[1];
	if (D != Dw)
		return fail(MOE_ERR_INVALID, "moe_ffn_forward: input rows of %lld, experts take %lld",
			    (long long)D, (long long)Dw);
	if ((int64_t)gate_inp->dim[0] != NE || (int64_t)gate_inp->dim[1] != D)
		return fail(MOE_ERR_INVALID, "moe_ffn_forward: router is [%llu,%llu], want [%lld,%lld]",
			    (unsigned long long)gate_inp->dim[0], (unsigned long long)gate_inp->dim[1],
			    (long long)NE, (long long)D);
	if (output->maxcap < (uint64_t)(T * D) && !(flags & MOE_DEVICE_IO))
		return fail(MOE_ERR_INVALID, "moe_ffn_forward: output too small");
	return MOE_OK;
}

// the forward of a cached layer: device pointers as given (MOE_DEVICE_IO),
// else the tokens copied in from the host and the output copied back
int forward_io(moe_layer *L, const moe_tensor_t *input, moe_tensor_t *output, int flags)
{
	const int64_t T = (int64_t)input->dim[0], D = (int64_t)input->dim[1];
	if (flags & MOE_DEVICE_IO)
		return moe_layer_forward(L, input->data, output->data, T, flags, nullptr);
	const size_t xb = align_up(T * D * 4, 256);
	if (int rc = ensure_dev_io(2 * xb))
		return rc;
	float *dx = (float *)g.dev_io, *dy = (float *)((char *)g.dev_io + xb);
	CK(cudaMemcpyAsync(dx, input->data, T * D * 4, cudaMemcpyHostToDevice, g.stream));
	if (int rc = moe_layer_forward(L, dx, dy, T, flags, nullptr))
		return rc;
	CK(cudaMemcpyAsync(output->data, dy, T * D * 4, cudaMemcpyDeviceToHost, g.stream));
	// the layer's error word comes back with the output (T == 0 runs nothing)
	if (T > 0)
		CK(cudaMemcpyAsync(g.err_pin, L->err, 4, cudaMemcpyDeviceToHost, g.stream));
	CK(cudaStreamSynchronize(g.stream));
	return T > 0 ? take_error(L, *g.err_pin) : MOE_OK;
}

int forward_common(const moe_tensor_t *input, moe_tensor_t *output, const moe_tensor_t *gate_inp,
		   int qtype, int64_t NE, int64_t F, int64_t Dw, const std::vector<const void *> &hg,
		   const std::vector<const void *> &hu, const std::vector<const void *> &hd,
		   size_t gbytes, size_t dbytes, size_t topk, int flags, moe_layer **used)
{
	if (int rc = check_io(input, output, gate_inp, NE, Dw, flags))
		return rc;
	const int64_t D = Dw;
	if (int rc = ensure_init())
		return rc;
	// resolve device weights (upload on first sight)
	const void *dr;
	if (int rc = resolve(gate_inp->data, (size_t)NE * D * 4, &dr))
		return rc;
	std::vector<const void *> dg(NE), du(NE), dd(NE);
	for (int64_t e = 0; e < NE; e++) {
		if (int rc = resolve(hg[e], gbytes, &dg[e]))
			return rc;
		if (int rc = resolve(hu[e], gbytes, &du[e]))
			return rc;
		if (int rc = resolve(hd[e], dbytes, &dd[e]))
			return rc;
	}
	std::vector<uintptr_t> key{(uintptr_t)gate_inp->data, (uintptr_t)qtype, (uintptr_t)NE,
				   (uintptr_t)F, (uintptr_t)topk, (uintptr_t)D};
	for (int64_t e = 0; e < NE; e++) {
		key.push_back((uintptr_t)hg[e]);
		key.push_back((uintptr_t)hu[e]);
		key.push_back((uintptr_t)hd[e]);
	}
	moe_layer *L;
	auto it = g.layers.find(key);
	if (it != g.layers.end()) {
		L = it->second;
	} else {
		moe_layer_desc desc{};
		desc.d_model = D;
		desc.d_ff = F;
		desc.n_experts = NE;
		desc.top_k = (int64_t)topk;
		desc.qtype = qtype;
		desc.flags = 0;
		desc.router_w = (const float *)dr;
		desc.router_bias = nullptr;
		desc.gate = dg.data();
		desc.up = du.data();
		desc.down = dd.data();
		if (int rc = moe_layer_create(&L, &desc))
			return rc;
		g.layers[key] = L;
	}
	if (used)
		*used = L;
	return forward_io(L, input, output, flags);
}

}  // namespace

extern "C" {

int moe_ffn_forward(const moe_tensor_t *input, moe_tensor_t *output, const moe_tensor_t *gate_inp,
		    const moe_tensor_t *gate_exps, const moe_tensor_t *up_exps,
		    const moe_tensor_t *down_exps, size_t topk, int flags)
{
	if (!gate_exps || !up_exps || !down_exps)
		return fail(MOE_ERR_INVALID, "moe_ffn_forward: null expert tensor");
	if (gate_exps->ndim != 3 || up_exps->ndim != 3 || down_exps->ndim != 3)
		return fail(MOE_ERR_INVALID, "moe_ffn_forward: expert tensors must be 3-D");
	// gate/up share a type; down may differ (K-quant files mix Q4_K and Q6_K)
	const int tgu = gate_exps->type, tdn = down_exps->type;
	if (up_exps->type != tgu || (tdn != tgu && !(ktype(tgu) && ktype(tdn))))
		return fail(MOE_ERR_UNSUPPORTED, "moe_ffn_forward: mixed expert dtypes");
	const int qt = tdn == tgu ? tgu : MOE_QTYPE2(tgu, tdn);
	const int64_t NE = (int64_t)gate_exps->dim[0], F = (int64_t)gate_exps->dim[1];
	const int64_t D = (int64_t)gate_exps->dim[2];
	if ((int64_t)up_exps->dim[0] != NE || (int64_t)up_exps->dim[1] != F ||
	    (int64_t)up_exps->dim[2] != D || (int64_t)down_exps->dim[0] != NE ||
	    (int64_t)down_exps->dim[1] != D || (int64_t)down_exps->dim[2] != F)
		return fail(MOE_ERR_INVALID, "moe_ffn_forward: expert shapes disagree");
	if (!legacy_type(tgu) && !ktype(tgu))
		return fail(MOE_ERR_UNSUPPORTED, "moe_ffn_forward: expert dtype %d", tgu);
	// repeat call with the same tensors: the cached layer, without
	// resolving every expert's view again (~200 lookups and a 198-entry key)
	const std::array<uintptr_t, 9> fk{(uintptr_t)(gate_inp ? gate_inp->data : nullptr),
					 (uintptr_t)gate_exps->qdata, (uintptr_t)up_exps->qdata,
					 (uintptr_t)down_exps->qdata, (uintptr_t)qt, (uintptr_t)NE,
					 (uintptr_t)F, (uintptr_t)D, (uintptr_t)topk};
	if (g.init) {
		auto ft = g.ffn_fast.find(fk);
		if (ft != g.ffn_fast.end()) {
			if (int rc = check_io(input, output, gate_inp, NE, D, flags))
				return rc;
			return forward_io(ft->second, input, output, flags);
		}
	}
	// tensor_at_q (olmoe.c:20-60): expert e starts e*rows*(cols/32)*bsz bytes in
	const size_t gb = (size_t)(F * qrow_bytes(tgu, D)), db = (size_t)(D * qrow_bytes(tdn, F));
	if (int rc = ensure_init())
		return rc;
	const void *tmp;
	// register each 3-D tensor as one range so every expert view resolves into it
	if (int rc = resolve(gate_exps->qdata, gb * NE, &tmp))
		return rc;
	if (int rc = resolve(up_exps->qdata, gb * NE, &tmp))
		return rc;
	if (int rc = resolve(down_exps->qdata, db * NE, &tmp))
		return rc;
	std::vector<const void *> hg(NE), hu(NE), hd(NE);
	for (int64_t e = 0; e < NE; e++) {
		hg[e] = (const char *)gate_exps->qdata + e * gb;
		hu[e] = (const char *)up_exps->qdata + e * gb;
		hd[e] = (const char *)down_exps->qdata + e * db;
	}
	moe_layer *L = nullptr;
	const int rc = forward_common(input, output, gate_inp, qt, NE, F, D, hg, hu, hd, gb, db, topk,
				      flags, &L);
	if (L)
		g.ffn_fast[fk] = L;
	return rc;
}

int moe_ffn_forward_split(const moe_tensor_t *input, moe_tensor_t *output,
			  const moe_tensor_t *gate_inp, const moe_tensor_t *const *gate_exp,
			  const moe_tensor_t *const *up_exp, const moe_tensor_t *const *down_exp,
			  size_t n_experts, size_t topk, int flags)
{
	if (!gate_exp || !up_exp || !down_exp || n_experts == 0)
		return fail(MOE_ERR_INVALID, "moe_ffn_forward_split: no experts");
	const int tgu = gate_exp[0]->type, tdn = down_exp[0] ? down_exp[0]->type : tgu;
	const int64_t F = (int64_t)gate_exp[0]->dim[0], D = (int64_t)gate_exp[0]->dim[1];
	if ((!legacy_type(tgu) && !ktype(tgu)) || (tdn != tgu && !(ktype(tgu) && ktype(tdn))))
		return fail(MOE_ERR_UNSUPPORTED, "moe_ffn_forward_split: expert dtypes %d/%d", tgu,
			    tdn);
	const int qt = tdn == tgu ? tgu : MOE_QTYPE2(tgu, tdn);
	std::vector<const void *> hg(n_experts), hu(n_experts), hd(n_experts);
	for (size_t e = 0; e < n_experts; e++) {
		const moe_tensor_t *a = gate_exp[e], *b = up_exp[e], *c = down_exp[e];
		if (!a || !b || !c || a->type != tgu || b->type != tgu || c->type != tdn ||
		    (int64_t)a->dim[0] != F || (int64_t)a->dim[1] != D || (int64_t)b->dim[0] != F ||
		    (int64_t)b->dim[1] != D || (int64_t)c->dim[0] != D || (int64_t)c->dim[1] != F)
			return fail(MOE_ERR_INVALID, "moe_ffn_forward_split: expert %zu shape/type", e);
		hg[e] = a->qdata;
		hu[e] = b->qdata;
		hd[e] = c->qdata;
	}
	const size_t gb = (size_t)(F * qrow_bytes(tgu, D)), db = (size_t)(D * qrow_bytes(tdn, F));
	return forward_common(input, output, gate_inp, qt, (int64_t)n_experts, F, D, hg, hu, hd, gb,
			      db, topk, flags, nullptr);
}

}  // extern "C"
