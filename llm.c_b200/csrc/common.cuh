// common.cuh — shared device helpers for the B200 MoE FFN kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define QK 32            // elements per Q8_0 / Q4_0 block (quant.h:11)
#define Q8_0_BYTES 34    // {fp16 d; int8 qs[32]}      (quant.h:14-17)
#define Q4_0_BYTES 18    // {fp16 d; uint8 qs[16]}     (quant.h:20-23)

namespace moe {

// Raise a kernel's dynamic shared-memory limit once per device and kernel
// (the attribute belongs to the device's context and persists), remembering
// what was set.
inline cudaError_t ensure_smem_ptr(const void *fn, size_t bytes)
{
	static const void *keys[256];
	static int devs[256];
	static size_t vals[256];
	static int used = 0;
	int dev = 0;
	cudaError_t e = cudaGetDevice(&dev);
	if (e != cudaSuccess)
		return e;
	int i = 0;
	for (; i < used; i++)
		if (keys[i] == fn && devs[i] == dev)
			break;
	if (i < used && bytes <= vals[i])
		return cudaSuccess;
	e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
	if (e != cudaSuccess)
		return e;
	if (i == used && used < 256) {
		keys[used] = fn;
		devs[used++] = dev;
	}
	if (i < 256)
		vals[i] = bytes;
	return cudaSuccess;
}

template <typename F>
inline cudaError_t ensure_smem(F *fn, size_t bytes)
{
	return ensure_smem_ptr(reinterpret_cast<const void *>(fn), bytes);
}

// SMs of the current device (cached per device)
inline int sm_count()
{
	static int n[64];
	int dev = 0;
	cudaGetDevice(&dev);
	if (dev < 0 || dev >= 64)
		dev = 0;
	if (!n[dev]) {
		int v = 0;
		cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
		n[dev] = v > 0 ? v : 148;
	}
	return n[dev];
}

enum QType { kF32 = 0, kQ8_0 = 1, kQ4_0 = 2, kQ4_K = 3, kQ6_K = 5 };

__host__ __device__ inline int64_t block_bytes(int qtype)
{
	return qtype == kQ8_0 ? Q8_0_BYTES : Q4_0_BYTES;
}

__host__ __device__ inline int64_t row_bytes(int qtype, int64_t cols)
{
	return cols / QK * block_bytes(qtype);
}

__device__ __forceinline__ float half_bits_to_float(uint16_t h)
{
	return __half2float(__ushort_as_half(h));
}

// exp(x) rounded once to fp32: evaluated in double precision and rounded,
// which is the correctly rounded result except within ~2^-29 ulp of a
// rounding midpoint.  glibc's expf (used by the reference, nn.c:475 and
// vector_avx512.h:50-63) is accurate to about 0.502 ulp, so the two agree
// except in rare near-midpoint cases.
__device__ __forceinline__ float exp_rn(float x)
{
	return (float)exp((double)x);
}

// reference's vector_reduce_sum (vector_avx512.h:127-134 for 16 lanes,
// vector_avx2.h:130-136 for 8): repeatedly add the upper half of the live
// lanes onto the lower half.  Lanes live in consecutive threads of a
// warp (lane index = threadIdx % lanes); the result is valid in lane 0.
// `__shfl_down_sync(v, s)` gives lane j the value of lane j+s.
template <int LANES>
__device__ __forceinline__ float lane_tree_sum(float v)
{
#pragma unroll
	for (int s = LANES / 2; s >= 1; s /= 2) {
		float o = __shfl_down_sync(0xffffffffu, v, s, LANES);
		v = __fadd_rn(v, o);
	}
	return v;
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
	for (int s = 16; s >= 1; s /= 2)
		v += __shfl_xor_sync(0xffffffffu, v, s);
	return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
	for (int s = 16; s >= 1; s /= 2)
		v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, s));
	return v;
}

// Programmatic dependent launch: a kernel launched with
// cudaLaunchAttributeProgrammaticStreamSerialization may start while the
// kernel before it on the stream is still running; it must not read that
// kernel's output (or write what it reads) before griddep_wait() returns,
// which waits for the earlier grid's completion and memory flush.  Without
// the attribute both are no-ops.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents()
{
	asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// silu(g) * u exactly as nn.c:475-478 computes it: g / (1 + exp(-g)) * u,
// each operation rounded once.
__device__ __forceinline__ float swiglu(float g, float u)
{
	float den = __fadd_rn(1.0f, exp_rn(-g));
	return __fmul_rn(__fdiv_rn(g, den), u);
}

}  // namespace moe
