// kernels.h — launchers shared between the kernel files and the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <cuda_fp16.h>

struct moe_layer;  // include/moe_b200.h

namespace moe {

// router.cu ------------------------------------------------------------
cudaError_t launch_router(const float *x, const float *w, const float *bias, int T, int d,
			  int NE, int K, int lanes, int mode_exact, int renorm, float *logits,
			  int32_t *ids, float *wts, float *probs, cudaStream_t st);
cudaError_t launch_router_logits(const float *x, const float *w, int T, int d, int NE, int lanes,
				 float *logits, cudaStream_t st);
// exact tiled router for d % 256 == 0 and NE % 16 == 0; also writes the
// fp16 hi/lo split of x (x16 may be NULL; q4 = Q4_0 block permutation)
bool router_tiled_ok(int d, int NE);
cudaError_t launch_router_tiled(const float *x, const float *w, int T, int d, int NE, int lanes,
				float *logits, __half *x16, int q4, cudaStream_t st);
cudaError_t launch_router_topk(const float *logits, const float *bias, int T, int NE, int K,
			       int lanes, int mode_exact, int renorm, int32_t *ids, float *wts,
			       float *probs, cudaStream_t st);
// dispatch also zeroes work[0..1] (the error word is sticky: the host
// reads and clears it)
cudaError_t launch_dispatch(const int32_t *ids, int npairs, int NE, int first, int nlocal,
			    int32_t *counts, int32_t *offsets, int32_t *perm, int32_t *pos_of,
			    int32_t *active, int32_t *n_active, int32_t *err, int32_t *work,
			    cudaStream_t st);
// one token: logits (one CTA per expert), then top-k and dispatch by the
// last CTA; cnt is a zeroed device counter (left zero)
bool router_t1_ok(int d, int NE, int K);
cudaError_t launch_router_t1(const float *x, const float *w, const float *bias, int d, int NE,
			     int K, int lanes, int mode_exact, int renorm, float *logits,
			     int32_t *ids, float *wts, int32_t *counts, int32_t *offsets,
			     int32_t *perm, int32_t *pos_of, int32_t *active, int32_t *n_active,
			     int32_t *err, int32_t *work, unsigned *cnt, cudaStream_t st);
// top-k + dispatch in one CTA (needs route_small_smem(T, NE, K) <= ~200 KB)
size_t route_small_smem(int T, int NE, int K);
cudaError_t launch_route_small(const float *logits, const float *bias, int T, int NE, int K,
			       int lanes, int mode_exact, int renorm, int first, int nlocal,
			       int32_t *ids, float *wts, int32_t *counts, int32_t *offsets,
			       int32_t *perm, int32_t *pos_of, int32_t *active, int32_t *n_active,
			       int32_t *err, int32_t *work, cudaStream_t st);

// experts.cu -----------------------------------------------------------
// Grouped expert GEMV over the expert segments given by counts/offsets.
// For the segment of expert e (positions off..off+n-1 of perm order):
//   in  row of position pos: in_perm  ? in[(perm[pos] / K)] : in[pos]
//   out row of position pos: out_perm ? out[perm[pos]]      : out[pos]
//   dual = 1: out[row][r] = swiglu(W1[e] row r . in, W2[e] row r . in)
//   dual = 0: out[row][r] = W1[e] row r . in
struct GemvArgs {
	const void *const *w1;  // device array [NE] of device pointers
	const void *const *w2;  // dual only
	int qtype;
	int rows, cols;         // weight matrix [rows, cols]
	int NE, K;
	int first_expert, n_local;  // experts computed here
	const int32_t *counts, *offsets, *perm;
	int in_perm, out_perm;
	const float *in;        // [*, cols]
	float *out;             // [*, rows]
	int dual;
	int tok;                // tokens per pass (set by the launcher)
};
cudaError_t launch_expert_gemv(const GemvArgs &a, cudaStream_t st);

// gemv.cu: y[rows] = W[rows, cols] . x[cols] for one activation row (see the
// file): the bulk-copy tensor-core kernel for cols % 256 == 0 and 16-byte
// aligned W, else one warp per row (cols % 64 == 0, 4-byte aligned W);
// 16-byte aligned x.  err (may be NULL) is set to 2 if a bounded wait expires.
bool gemv1_supported(int qtype, int64_t rows, int64_t cols, uintptr_t w, uintptr_t x, uintptr_t y);
// pdl: launched as a programmatic dependent of the kernel before it (the
// weights stream at once; x is read after that kernel completes)
cudaError_t launch_gemv1(const void *w, int qtype, int64_t rows, int64_t cols, const float *x,
			 float *y, int32_t *err, cudaStream_t st, bool pdl = false);
// the tensor-core GEMV with its x made in the prologue from the residual
// stream: h = hidden + delta (delta may be NULL), x = rms_norm(h) * weight;
// CTA 0 stores h into hidden_out (not hidden: the other CTAs still read it)
struct NormIn {
	const float *hidden = nullptr, *delta = nullptr, *weight = nullptr;
	float *hidden_out = nullptr;
	float eps = 1e-5f;
};
bool gemv_norm_supported(int qtype, int64_t cols, uintptr_t w);

// gemv.cu: the experts of ONE token (moe_layer_forward at T = 1) through the
// single-row GEMV: the matrices of the token's K slots are row segments of
// one launch, read in column chunks.  gate/up: segments gate of slots
// 0..K-1 then up of slots 0..K-1, all against the token x; down: segment k
// = the down matrix of slot k against h_k = swiglu(gate_k, up_k).
struct SegMap {
	const void *const *wtab = nullptr;  // NULL: a plain GEMV; else device [3][NE]
	const int32_t *ids = nullptr;       // device [K]: the token's experts, slot order
	int NE = 0, K = 0, down = 0;
	int nchunks = 1;                    // column chunks per row
	int64_t rb_full = 0;                // bytes of a whole matrix row
	const float *gu = nullptr;          // down: gate/up results [2K][cols]
	float *part = nullptr;              // [nchunks][segments][rows] partial row sums
};
// 0 when the shapes (d_model D, d_ff F) do not fit; else the down matrix's
// column chunks
int expert_t1_chunks(int qtype, int64_t D, int64_t F, int K);
// ids (the token's K experts) and w (their weights) on the device; gu:
// [2K][F] and part: [chunks][K][D] scratch; out: [D].  stage 0: gate/up
// (gu), 1: down (part), 2: combine (out)
cudaError_t launch_expert_t1(int stage, const void *const *wtab, const int32_t *ids,
			     const float *w, int qtype, int64_t D, int64_t F, int NE, int K,
			     const float *x, float *gu, float *part, float *out, int32_t *err,
			     cudaStream_t st);
cudaError_t launch_gemv_norm(const void *w, int qtype, int64_t rows, int64_t cols,
			     const NormIn &nin, float *y, int32_t *err, bool pdl, cudaStream_t st);

// expert_mma.cu: tensor-core grouped expert GEMV (decode).  Same segment
// semantics as GemvArgs; activations are fp16 hi/lo rows [row][2][cols]
// (Q4_0: each 32-element block stored in the permuted order of q4_slot).
struct MmaArgs {
	const void *const *w1;
	const void *const *w2;
	int qtype;
	int rows, cols;
	int NE, K;
	int first_expert, n_local;
	const int32_t *counts, *offsets, *perm;
	int in_perm, out_perm;
	const __half *in16;     // [*, 2, cols]
	float *out;             // single: [*, rows] fp32
	__half *out16;          // dual:   [*, 2, rows] fp16 hi/lo
	int dual;
	int32_t *err;           // set to 2 when a bounded wait expires
	const int32_t *active;  // [n_active] experts with work, ascending
	const int32_t *n_active;
	int32_t *work;          // item counter, zero at launch (dispatch zeroes it)
};
bool expert_mma_supported(int qtype, int cols);
cudaError_t launch_expert_mma(const MmaArgs &a, cudaStream_t st);
cudaError_t launch_split_f16(const float *x, int64_t rows, int cols, int qtype, __half *out,
			     cudaStream_t st);

// decode.cu: the whole layer of a decode-sized batch in one cooperative
// kernel (router, routing, gate/up, down, combine).
struct DecodeArgs {
	const float *x;            // [T, D]
	const float *router_w;     // [NE, D]
	const float *router_bias;  // [NE] or NULL
	const void *const *dptrs;  // device [3][NE]: gate, up, down weight pointers
	int T, D, F, NE, K;
	int mode_exact, renorm;
	float *logits;             // [T, NE]
	__half *x16;               // [T, 2, D]
	__half *h16;               // [pairs, 2, F]
	float *Y;                  // [T*K, D]
	float *out;                // [T, D]
	int32_t *ids;              // [T*K]
	float *wts;                // [T*K]
	int32_t *counts, *offsets, *perm, *active, *n_active;
	// sticky error word (the host reads and clears it): 1 expert id out of
	// range, 2 bounded mbarrier wait expired, 3 grid barrier expired,
	// 4 expert-parallel exchange wait expired, 5 ranks passed different T
	int32_t *err;
	unsigned long long *gbar;  // grid barrier state (decode_barrier_bytes), zero when allocated
	uint64_t *stamps;          // NULL or [grid][decode_stamps()] phase times (ns)
	// expert parallelism (world > 1): this GPU computes experts
	// [first_expert, first_expert + n_local).
	//   shard = 0 (replicated tokens): every rank has the same T tokens; each
	//     (token, slot) row of the local experts goes to every rank's
	//     exchange buffer and every rank combines all rows in slot order.
	//   shard = 1 (token-sharded): x holds this rank's own T tokens (every
	//     rank passes the same T).  Each rank writes its tokens (fp16 hi/lo)
	//     and top-k ids into every rank's exchange buffer; after the
	//     cross-rank arrival each rank dispatches the pairs of all world*T
	//     tokens to its local experts, and every row it produces goes to the
	//     exchange buffer of the rank that owns the token; each rank then
	//     combines its own tokens.
	int first_expert, n_local;
	int rank, world, shard;
	float *const *ybuf;        // device [world]: exchange buffers (two Y halves each)
	int64_t ybuf_half;         // floats from one half to the other
	unsigned long long *const *inbound;  // device [world]: rank r's row-arrival counters
	unsigned long long *const *routed;   // device [world]: rank r's routing-arrival counters
	__half *const *xg;         // device [world]: gathered tokens [world*T][2][D] (shard)
	int32_t *const *idg;       // device [world]: T of each rank [16], then ids [world*T*K]
	unsigned long long *launches;        // this rank's count of expert-parallel launches
	unsigned long long *shard_launches;  // ... of token-sharded ones (the routing arrivals)
	uint64_t ep_wait_ns;       // limit of the cross-rank waits (0: the 2 s default)
};
constexpr int kMaxEpRanks = 8;
constexpr int kEpFlagStride = 16;  // u64s (128 bytes) per counter
constexpr int kEpIdsHeader = 16;   // int32 slots before the gathered ids
// kernel-side limits of the fused decode kernel
constexpr int kDecodeMaxT = 64;           // tokens per rank
constexpr int kDecodeMaxPairs = 1024;     // this rank's (token, slot) pairs
constexpr int kDecodeMaxPairsAll = 2048;  // every rank's pairs (token-sharded)
// exchange buffer of one rank (one allocation, shared by CUDA IPC):
//   Y halves      2 * y_half floats
//   counters      inbound[kMaxEpRanks], routed[kMaxEpRanks], launches,
//                 token-sharded launches (one 128-byte line each)
//   gathered ids  kEpIdsHeader + kMaxEpRanks * kDecodeMaxPairs int32
//   gathered x    kMaxEpRanks * kDecodeMaxT rows of 2 * D halves
struct EpLayout {
	size_t inbound, routed, launches, shard_launches, idg, xg, bytes;
};
inline EpLayout ep_layout(int64_t y_half, int64_t D)
{
	EpLayout l;
	const size_t line = (size_t)kEpFlagStride * 8;
	l.inbound = (size_t)(2 * y_half) * 4;
	l.inbound = (l.inbound + 255) / 256 * 256;
	l.routed = l.inbound + kMaxEpRanks * line;
	l.launches = l.routed + kMaxEpRanks * line;
	l.shard_launches = l.launches + line;
	l.idg = l.shard_launches + line;
	l.xg = l.idg + (size_t)(kEpIdsHeader + kMaxEpRanks * kDecodeMaxPairs) * 4;
	l.xg = (l.xg + 255) / 256 * 256;
	l.bytes = l.xg + (size_t)kMaxEpRanks * kDecodeMaxT * 2 * D * 2;
	return l;
}
// world_pairs: the (token, slot) pairs of every rank the kernel dispatches
// (T*K, or world*T*K when token-sharded)
bool decode_supported(int qtype, int64_t T, int D, int F, int NE, int K, int64_t world_pairs,
		      uintptr_t x, uintptr_t router_w, uintptr_t out);
int decode_stamps();
int decode_max_t();
size_t decode_barrier_bytes(int ctas);
void decode_stage_ends(int *ends);
cudaError_t launch_decode_layer(const DecodeArgs &a, int qtype, int lanes, cudaStream_t st);

// expert_gemm.cu: prefill-sized grouped GEMM on tcgen05 (see the file).
// Segment semantics as MmaArgs; activations are fp16 hi/lo rows in pair
// order, natural column order: in16 [in_rows][2][cols].  maps1/maps2 are device
// arrays of per-expert weight tensor maps (encode_weight_map), indexed by
// the global expert id.
struct GemmArgs {
	const void *maps1;       // W1 (gate, or down) tensor maps [NE]
	const void *maps2;       // dual: W2 (up) tensor maps [NE]
	int qtype;
	int rows, cols;          // weight matrix; rows % 128 (dual) / 256, cols % 256
	int n_local;
	const int32_t *counts, *offsets, *perm;
	const int32_t *active, *n_active;
	int out_perm;
	const __half *in16;
	__half *out16;           // dual: [pairs][2][rows] swiglu as fp16 hi/lo
	float *out;              // single: [pairs][rows]
	int dual;
	int32_t *err;
};
bool expert_gemm_supported(int qtype, int rows, int cols, int dual);
// one weight matrix (rows x cols, GGUF blocks, 16-byte aligned) as the tensor
// map the GEMM reads raw chunks through; map points at weight_map_bytes()
bool encode_weight_map(void *map, const void *w, int qtype, int rows, int cols);
size_t weight_map_bytes();
cudaError_t launch_expert_gemm(const GemmArgs &a, int64_t in_rows, cudaStream_t st);
// out[pos] = fp16 hi/lo of x[perm[pos] / K] (pair order, natural columns)
cudaError_t launch_gather_split(const float *x, const int32_t *perm, int64_t pairs, int cols,
				int K, __half *out, cudaStream_t st);

// out[t, :] = sum_s Y[t*K + s, :] / (1 / w[t*K + s]) in slot order
cudaError_t launch_combine(const float *Y, const float *w, int T, int K, int d, float *out,
			   cudaStream_t st);

// the same with the rows of Y at the pairs' dispatch positions:
// Y[pos_of[t*K + s]] (d % 4 == 0, Y and out 16-byte aligned)
cudaError_t launch_combine_pos(const float *Y, const int32_t *pos_of, const float *w, int T, int K,
			       int d, float *out, cudaStream_t st);

// rows moved by segment: seg [nseg][3] = (source-major row, expert-major
// row, rows) on the device; dir 0: source-major -> expert-major, 1: back
cudaError_t launch_copy_segments(const void *src, void *dst, const int64_t *seg, int nseg, int dir,
				 int64_t row_bytes, cudaStream_t st);

// ret[i] = ret[i] + add[i % n_add]  (bias of tensor_mma_transposed_2x2)
cudaError_t launch_add_bias(float *ret, const float *add, int64_t total, int64_t n_add,
			    cudaStream_t st);

// kquant.cu: K-quant experts (Q4_K = 3, Q6_K = 5, the reference's tensor
// dtype values) over the dispatch's expert segments
struct KqArgs {
	const void *const *w1, *const *w2;  // device arrays [NE] of expert matrices
	int rows, cols;                     // the matrices' shape (cols % 256 == 0)
	int K, first_expert, n_local;
	const int32_t *counts, *offsets, *perm;
	const uint8_t *x8;                  // gate/up: tokens as Q8_K [T][cols/256]
	const float *hin;                   // down: h rows [pairs][cols]
	float *h;                           // gate/up: h rows [pairs][rows] (pair order)
	float *out;                         // down: Y rows [pairs by t*K + slot][rows]
};
bool kquant_type(int qtype);
cudaError_t launch_quantize_q8k(const float *x, int T, int D, uint8_t *y, cudaStream_t st);
cudaError_t launch_kq_gate_up(const KqArgs &a, int qtype, cudaStream_t st);
cudaError_t launch_kq_down(const KqArgs &a, int qtype, cudaStream_t st);

// capi.cu: the dense projection y[m, rows] = x[m, cols] . W[rows, cols]^T
// (Q8_0/Q4_0 W) behind moe_gemv_device, with caller-owned scratch; returns
// a MOE_* status (the message through moe_last_error)
struct DenseScratch {
	void *meta = nullptr;
	__half *x16 = nullptr;
	size_t x16_bytes = 0;
};
int dense_forward(DenseScratch &s, const void *w, int qtype, int64_t rows, int64_t cols,
		  const float *x, int64_t m, float *y, int32_t *err, cudaStream_t st);
void dense_scratch_free(DenseScratch &s);
void set_last_error(const char *msg);
// rows a MoE layer's scratch holds (it only grows; buffers move when it does)
int64_t layer_scratch_rows(const ::moe_layer *L);
int ensure_library();
cudaStream_t library_stream();

// model.cu: the transformer around the MoE layers --------------------------
// hidden[t] = dequant(wte row tok[t]); out[t] = rms_norm(hidden[t]) * w
// (err |= 1 for a token id outside [0, V))
cudaError_t launch_embed_norm(const void *wte, int wtype, int64_t V, int E, const int32_t *tok,
			      int T, const float *w, float eps, float *hidden, float *out,
			      int32_t *err, cudaStream_t st, bool pdl = false);
// hidden[t] += delta[t]; out[t] = rms_norm(hidden[t]) * w
cudaError_t launch_add_norm(float *hidden, const float *delta, const float *w, int T, int E,
			    float eps, float *out, cudaStream_t st, bool pdl = false);
// per token: q (and k) RMS-normed over the whole vector (qk_norm), RoPE on
// the pairs (2i, 2i+1) of each head from the cos/sin table rope[pos][i];
// q -> q_out [T, H*HL], k and v -> the layer's cache at rows size + t
struct QkvArgs {
	const float *qkv;          // [T, (H + 2 KVH) * HL]
	const float *q_norm, *k_norm;  // [H*HL], [KVH*HL] or NULL (no QK-norm)
	const float2 *rope;        // [C][HL/2] (cos, sin)
	const int32_t *pos;        // [T]
	const int32_t *size;       // cache rows already filled (device scalar)
	float *q_out;              // [T, H*HL]
	float *kc, *vc;            // this layer's cache [KVH][C][HL]
	int T, H, KVH, HL, C;
	float eps;
	int32_t *err;              // err |= 2: position or cache row out of range
};
cudaError_t launch_qk_rope(const QkvArgs &a, cudaStream_t st);
// causal attention of q [T, H*HL] over the cache rows [0, size + T) of this
// layer (query t sees rows <= size + t); GQA: query head h reads kv head
// h / (H / KVH).  T == 1 splits the rows into kAttnChunk-row chunks (part:
// [H][attn_splits(C)][HL + 2] scratch) and merges them.
constexpr int kAttnChunk = 64;
inline int attn_splits(int C) { return (C + kAttnChunk - 1) / kAttnChunk; }
// CTAs per head of the one-launch decode step (balanced row ranges)
inline int attn_step_splits(int C) { return C < 16 ? C : 16; }   // <= 16: the merge's reach
cudaError_t launch_attention(const float *q, const float *kc, const float *vc, const int32_t *size,
			     int T, int H, int KVH, int HL, int C, float scale_div, float *part,
			     float *out, cudaStream_t st);
// T = 1: QK-norm + RoPE of the step's q and k, the new cache row and the
// split attention with the merge by each head's last CTA, in one launch
struct AttnStepArgs {
	const float *qkv;              // [(H + 2 KVH) * HL]
	const float *q_norm, *k_norm;  // or NULL
	const float2 *rope;
	const int32_t *pos, *size;     // device scalars
	float *kc, *vc;                // this layer's cache
	float *part;                   // [H][attn_step_splits(C)][HL + 2]
	int32_t *cnt;                  // [H] arrival counters, zero between launches
	float *out;                    // [H * HL]
	int H, KVH, C;
	float eps, scale_div;
	int32_t *err;
};
cudaError_t launch_attn_step(const AttnStepArgs &a, cudaStream_t st);
// launch with programmatic stream serialization (see griddep_wait), unless
// MOE_PDL=0 in the environment
bool pdl_enabled();

// greedy pick (main.c:189-193: the first maximum) of logits [V] into
// state[0] and picks[state[6] % pick_cap] (state[6] counts the picks); with
// advance, the decode state {tok, pos, size, model_pos} moves one row on
// (scratch: device, at least 4 KB, zero before the first call)
cudaError_t launch_argmax_advance(const float *logits, int V, int C, int32_t *state,
				  int32_t *picks, int pick_cap, int advance, float *scratch,
				  cudaStream_t st, bool pdl = false);
// cache rows [drop, drop + keep) -> [0, keep) of every layer, head, K and V
cudaError_t launch_kv_shift(float *kc, float *vc, int L, int KVH, int C, int HL, int keep,
			    int drop, cudaStream_t st);

// synth.cu -------------------------------------------------------------
cudaError_t launch_synth_gauss(float *dst, uint64_t stream_seed, uint64_t offset, int64_t n,
			       float sd, cudaStream_t st);
cudaError_t launch_quantize(const float *src, int64_t rows, int64_t cols, int qtype, void *dst,
			    cudaStream_t st);

}  // namespace moe
