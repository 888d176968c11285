// SPDX-License-Identifier: GPL-2.0-or-later
// Row operations of charsiu's decode step, used by its kernels (forward.cuh):
// the activation quantiser of one 32-block, 16-byte asynchronous copies, the
// ordered fp32 sum, and rmsnorm + quantiser by one CTA.
//
// (Running the rmsnorm inside each CTA of the matvec after it, instead of as
// a launch of its own, was measured slower on the 1B decode step: 1.035 ms a
// token against 0.688 ms. Every CTA then quantises the whole activation
// again, about a thousand times over, and the issue slots that costs exceed
// the launch and the global-memory round trip it saves.)
#pragma once

#include <cstdint>

#include "ptx.cuh"

namespace cgpu {

// charsiu_act_set of one 32-block held one element a lane (src/gguf.c:852-881):
// amax by max (order-free), d = amax / 127, q = round-to-nearest-even of
// v * (1 / d). Lane 0 writes d.
__device__ __forceinline__ void quantise_block_warp(float v, int lane, int8_t *q, float *d)
{
	float amax = fabsf(v);
	for (int o = 16; o; o >>= 1)
		amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
	const float dd = __fdiv_rn(amax, 127.0f);
	const float inv = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
	q[lane] = (int8_t)__float2int_rn(__fmul_rn(v, inv));
	if (lane == 0)
		*d = dd;
}

// 16-byte asynchronous copy global -> shared (LDGSTS), and the wait for all
// of this thread's
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem)
{
	const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
	asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all()
{
	asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// The sum a[0] + a[1] + ... + a[n-1] in order from 0.0f, one fp32 add at a
// time (the reference's `ss += x[i] * x[i]` once the squares are rounded, and
// its softmax sum), by ONE thread; a in shared memory, 16-byte aligned. The
// chain is n dependent adds; the loads run ahead of it in 16-byte words.
// Measured on B200 for 2048 terms: 9.4k cycles (4.6 a term). Slower forms
// measured: the terms held 64 a lane and the lanes adding in turn (12.6k),
// lane 0 taking every term by shuffle (17.8k), and an exact parallel form --
// jumping the running sum over whole runs of terms that keep it in one
// binade, where fl(s + a) is s plus a rounded to the binade's grid, with CTA
// prefix scans between the binade changes and ties -- about 2.1k cycles a
// round and 6 to 9 rounds (13k to 20k).
__device__ __forceinline__ float ordered_sum_seq(const float *a, uint32_t n)
{
	const float4 *a4 = reinterpret_cast<const float4 *>(a);
	float s = 0.0f;
	uint32_t i = 0;
#pragma unroll 16
	for (; i < n / 4; i++) {
		const float4 v = a4[i];
		s = __fadd_rn(s, v.x);
		s = __fadd_rn(s, v.y);
		s = __fadd_rn(s, v.z);
		s = __fadd_rn(s, v.w);
	}
	for (i *= 4; i < n; i++)
		s = __fadd_rn(s, a[i]);
	return s;
}

// rmsnorm (reference src/llama.c:316-326) of x (+ add), then the
// quantiser of the result into aq / ad, by the whole CTA: xs[i] = x[i] +
// add[i] (x alone when add is null), ss = the ordered sum of xs[i]^2 (thread
// 0), scale = 1 / sqrtf(ss / n + eps), v = xs[i] * scale * w[i] per element,
// one warp a 32-block. xs, sq, ws: n floats each of shared memory, 16-byte
// aligned, ws holding w already (copied in by the caller). *scale_sh: a
// shared float. Ends with a barrier; xs still holds x + add.
__device__ __forceinline__ void norm_quant_cta(const float *__restrict__ x,
					       const float *__restrict__ add, uint32_t n, float eps,
					       float *xs, float *sq, const float *ws, float *scale_sh,
					       int8_t *aq, float *ad)
{
	for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
		float v = x[i];
		if (add)
			v = __fadd_rn(v, add[i]);
		xs[i] = v;
		sq[i] = __fmul_rn(v, v);
	}
	cp_async_wait_all();
	__syncthreads();
	if (threadIdx.x == 0) {
		const float ss = ordered_sum_seq(sq, n);
		*scale_sh = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
	}
	__syncthreads();
	const float scale = *scale_sh;
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	for (uint32_t b = warp; b < n / 32; b += blockDim.x / 32) {
		const uint32_t i = b * 32 + lane;
		quantise_block_warp(__fmul_rn(__fmul_rn(xs[i], scale), ws[i]), lane, aq + b * 32,
				    ad + b);
	}
	__syncthreads();
}

} // namespace cgpu
