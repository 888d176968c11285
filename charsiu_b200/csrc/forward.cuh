// SPDX-License-Identifier: GPL-2.0-or-later
// The rest of charsiu's decode step on the device (reference
// src/llama.c:316-386 and 743-856): rmsnorm, the activation quantiser, RoPE
// and the KV cache, attention, SiLU and the residual adds -- every float
// operation in the reference's order and rounding, so a token's logits are
// the reference's bit for bit.
//
// What that costs on a GPU: the reference's sums are sequential fp32 chains
// (rmsnorm's sum of squares over n_embd, a score's dot over head_dim, the
// softmax's sum over positions, each output's sum over positions), so each
// chain runs in ONE thread, in order; the parallel work around it (products,
// maxima, quantisation) uses the rest of the CTA. And expf: the reference
// calls the host C library's expf, whose last bit a GPU's own exp does not
// reproduce, so exp_exact() looks the value up in a table of the host
// library's own results (built at open; see resident.cu).
#pragma once

#include <cstdint>

#include "ptx.cuh"

namespace cgpu {

// The host expf table covers |x| in [2^-26, 2^7): biased exponents 101..133,
// both signs, every mantissa. Below it expf rounds to 1; at and above 128 it
// is +inf (x > 0) or 0 (x < 0).
constexpr uint32_t EXPTAB_E0 = 101, EXPTAB_NE = 33;
constexpr uint64_t EXPTAB_ENTRIES = 2ull * EXPTAB_NE << 23;

// The step's small device inputs and outputs: the token, its position, and
// the argmax of its logits.
constexpr int FWD_IO_TOKEN = 0, FWD_IO_POS = 1, FWD_IO_NEXT = 2, FWD_IO_WORDS = 4;

__device__ __forceinline__ float exp_exact(float x, const float *__restrict__ tab)
{
	const uint32_t b = __float_as_uint(x);
	const uint32_t e = (b >> 23) & 0xffu, sign = b >> 31;
	if (e == 0xffu)
		return (b & 0x7fffffu) ? x : (sign ? 0.0f : x);      // NaN, -inf -> 0, +inf
	if (e < EXPTAB_E0)
		return 1.0f;
	if (e >= EXPTAB_E0 + EXPTAB_NE)
		return sign ? 0.0f : __int_as_float(0x7f800000);
	const uint64_t idx = ((uint64_t)(sign * EXPTAB_NE + (e - EXPTAB_E0)) << 23) | (b & 0x7fffffu);
	return tab[idx];
}

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

// x (+ add, written back to x when add is given), then rmsnorm with weights
// w (src/llama.c:316-326: ss += x*x in order, scale = 1 / sqrtf(ss / n + eps),
// out = x * scale * w), then the quantiser of the result. One CTA; n a
// multiple of 32, at most FWD_NORM_MAX. The sum of squares is one chain of n
// dependent adds in thread 0 (the squares and shared-memory loads sit off the
// chain); everything else is spread over the CTA.
constexpr uint32_t FWD_NORM_MAX = 8192;
constexpr int FWD_NORM_THREADS = 1024;

__global__ void __launch_bounds__(FWD_NORM_THREADS)
fwd_norm_quant_kernel(float *__restrict__ x, const float *__restrict__ add,
		      const float *__restrict__ w, uint32_t n, float eps, int8_t *__restrict__ q,
		      float *__restrict__ d)
{
	__shared__ float xs[FWD_NORM_MAX];
	__shared__ float scale_s;
	pdl_wait();
	for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
		float v = x[i];
		if (add) {
			v = __fadd_rn(v, add[i]);
			x[i] = v;
		}
		xs[i] = v;
	}
	__syncthreads();
	if (threadIdx.x == 0) {
		float ss = 0.0f;
#pragma unroll 16
		for (uint32_t i = 0; i < n; i++)
			ss = __fadd_rn(ss, __fmul_rn(xs[i], xs[i]));
		scale_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
	}
	__syncthreads();
	pdl_launch_dependents();
	const float scale = scale_s;
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	for (uint32_t b = warp; b < n / 32; b += blockDim.x / 32) {
		const uint32_t i = b * 32 + lane;
		const float v = __fmul_rn(__fmul_rn(xs[i], scale), w[i]);
		quantise_block_warp(v, lane, q + b * 32, d + b);
	}
}

// RoPE of q (n_head heads) and k (n_head_kv) at this token's position, with
// the (cos, sin) pairs of that position from a table the host filled with the
// reference's own libm calls (src/llama.c:364-383), then k and v into the
// layer's cache row of that position (src/llama.c:781-789).
__global__ void fwd_rope_kv_kernel(float *__restrict__ qv, float *__restrict__ kv,
				   const float *__restrict__ vv, const float *__restrict__ rope_cs,
				   const int *__restrict__ io, float *__restrict__ kcache,
				   float *__restrict__ vcache, uint32_t n_head, uint32_t n_head_kv,
				   uint32_t hd)
{
	pdl_wait();
	const uint32_t half = hd / 2, kvdim = n_head_kv * hd;
	const uint32_t pairs = (n_head + n_head_kv) * half;
	const int pos = io[FWD_IO_POS];
	const float *cs = rope_cs + (size_t)pos * hd;
	const size_t row = (size_t)pos * kvdim;
	for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < pairs; j += gridDim.x * blockDim.x) {
		const uint32_t hh = j / half, i = j % half;
		float *p = hh < n_head ? qv + hh * hd : kv + (hh - n_head) * hd;
		const float c = cs[2 * i], s = cs[2 * i + 1];
		const float x0 = p[2 * i], x1 = p[2 * i + 1];
		const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
		const float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
		p[2 * i] = y0;
		p[2 * i + 1] = y1;
		if (hh >= n_head) {
			const uint32_t off = (hh - n_head) * hd + 2 * i;
			kcache[row + off] = y0;
			kcache[row + off + 1] = y1;
		}
	}
	for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < kvdim; j += gridDim.x * blockDim.x)
		vcache[row + j] = vv[j];
	pdl_launch_dependents();
}

// One head of attention at this position (src/llama.c:792-817), then the
// quantiser of the head's outputs (head_dim a multiple of 32, so every
// 32-block of the attention output lies inside one head): scores
// a_t = (sum_i q_i k_ti, in order) * scale; softmax (the max, expf, the sum
// over t in order, the division); out_i = sum_t att_t v_ti in order from 0.
// One CTA a head. Each score's dot runs in one thread, the softmax sum in
// thread 0, each out_i in one thread.
constexpr int FWD_ATTN_THREADS = 256;

inline size_t fwd_attention_smem(uint32_t n_ctx, uint32_t hd)
{
	return ((size_t)n_ctx + 2 * hd) * sizeof(float);
}

__global__ void __launch_bounds__(FWD_ATTN_THREADS)
fwd_attention_kernel(const float *__restrict__ qv, const float *__restrict__ kcache,
		     const float *__restrict__ vcache, const int *__restrict__ io,
		     uint32_t n_head, uint32_t n_head_kv, uint32_t hd, uint32_t n_ctx, float scale,
		     const float *__restrict__ exptab, int8_t *__restrict__ q,
		     float *__restrict__ d)
{
	extern __shared__ __align__(16) float fsm[];
	float *att = fsm;                  // n_ctx scores
	float *qs = fsm + n_ctx;           // this head's q
	float *os = qs + hd;               // this head's outputs
	__shared__ float red[FWD_ATTN_THREADS / 32];
	__shared__ float sum_s;
	pdl_wait();
	const uint32_t h = blockIdx.x, kvdim = n_head_kv * hd;
	const uint32_t kvh = h / (n_head / n_head_kv);
	const int np = io[FWD_IO_POS] + 1;
	for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x)
		qs[i] = qv[h * hd + i];
	__syncthreads();
	const float *kh = kcache + kvh * hd, *vh = vcache + kvh * hd;
	for (int t = threadIdx.x; t < np; t += blockDim.x) {
		const float4 *kt = reinterpret_cast<const float4 *>(kh + (size_t)t * kvdim);
		float a = 0.0f;
		for (uint32_t i = 0; i < hd / 4; i++) {
			const float4 k4 = kt[i];
			a = __fadd_rn(a, __fmul_rn(qs[4 * i], k4.x));
			a = __fadd_rn(a, __fmul_rn(qs[4 * i + 1], k4.y));
			a = __fadd_rn(a, __fmul_rn(qs[4 * i + 2], k4.z));
			a = __fadd_rn(a, __fmul_rn(qs[4 * i + 3], k4.w));
		}
		att[t] = __fmul_rn(a, scale);
	}
	__syncthreads();
	// the max: any order gives the reference's value for NaN-free scores (a NaN
	// needs a non-finite weight or delta)
	float mx = -__int_as_float(0x7f800000);
	for (int t = threadIdx.x; t < np; t += blockDim.x)
		mx = fmaxf(mx, att[t]);
	for (int o = 16; o; o >>= 1)
		mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
	if ((threadIdx.x & 31) == 0)
		red[threadIdx.x >> 5] = mx;
	__syncthreads();
	mx = red[0];
	for (int wi = 1; wi < FWD_ATTN_THREADS / 32; wi++)
		mx = fmaxf(mx, red[wi]);
	for (int t = threadIdx.x; t < np; t += blockDim.x)
		att[t] = exp_exact(__fsub_rn(att[t], mx), exptab);
	__syncthreads();
	if (threadIdx.x == 0) {
		float s = 0.0f;
#pragma unroll 8
		for (int t = 0; t < np; t++)
			s = __fadd_rn(s, att[t]);
		sum_s = s;
	}
	__syncthreads();
	const float sum = sum_s;
	for (int t = threadIdx.x; t < np; t += blockDim.x)
		att[t] = __fdiv_rn(att[t], sum);
	__syncthreads();
	for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) {
		float o = 0.0f;
#pragma unroll 4
		for (int t = 0; t < np; t++)
			o = __fadd_rn(o, __fmul_rn(att[t], vh[(size_t)t * kvdim + i]));
		os[i] = o;
	}
	__syncthreads();
	pdl_launch_dependents();
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	for (uint32_t b = warp; b < hd / 32; b += blockDim.x / 32) {
		const uint32_t e = h * hd + b * 32;
		quantise_block_warp(os[b * 32 + lane], lane, q + e, d + e / 32);
	}
}

// SiLU(gate) * up (src/llama.c:831-836: g *= 1 / (1 + expf(-g)); g * up),
// then the quantiser of the result. One warp a 32-block.
__global__ void fwd_silu_quant_kernel(const float *__restrict__ gate, const float *__restrict__ up,
				      uint32_t n, const float *__restrict__ exptab,
				      int8_t *__restrict__ q, float *__restrict__ d)
{
	pdl_wait();
	const uint32_t b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
	const int lane = threadIdx.x & 31;
	if (b < n / 32) {
		const uint32_t i = b * 32 + lane;
		float g = gate[i];
		const float e = exp_exact(-g, exptab);
		g = __fmul_rn(g, __fdiv_rn(1.0f, __fadd_rn(1.0f, e)));
		quantise_block_warp(__fmul_rn(g, up[i]), lane, q + b * 32, d + b);
	}
	pdl_launch_dependents();
}

// llama_argmax (src/llama.c:860-868): the first index of the maximum, a NaN
// never taken past index 0 (and index 0 kept when it is NaN), into
// io[FWD_IO_NEXT]. One CTA: each thread the first maximum of its stride,
// then the CTA's (value, smallest index) reduction.
constexpr int FWD_ARGMAX_THREADS = 1024;

__global__ void __launch_bounds__(FWD_ARGMAX_THREADS)
fwd_argmax_kernel(const float *__restrict__ x, uint32_t n, int *__restrict__ io)
{
	__shared__ float rv[FWD_ARGMAX_THREADS / 32];
	__shared__ uint32_t ri[FWD_ARGMAX_THREADS / 32];
	pdl_wait();
	float bv = -__int_as_float(0x7f800000);
	uint32_t bi = 0xffffffffu;
	for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
		const float v = x[i];
		if (v > bv || (v == bv && bi == 0xffffffffu)) {
			bv = v;
			bi = i;
		}
	}
	for (int o = 16; o; o >>= 1) {
		const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
		const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
		if (oi != 0xffffffffu && (bi == 0xffffffffu || ov > bv || (ov == bv && oi < bi))) {
			bv = ov;
			bi = oi;
		}
	}
	if ((threadIdx.x & 31) == 0) {
		rv[threadIdx.x >> 5] = bv;
		ri[threadIdx.x >> 5] = bi;
	}
	__syncthreads();
	if (threadIdx.x == 0) {
		for (int w = 1; w < FWD_ARGMAX_THREADS / 32; w++)
			if (ri[w] != 0xffffffffu &&
			    (bi == 0xffffffffu || rv[w] > bv || (rv[w] == bv && ri[w] < bi))) {
				bv = rv[w];
				bi = ri[w];
			}
		const float x0 = x[0];
		io[FWD_IO_NEXT] = (x0 != x0 || bi == 0xffffffffu) ? 0 : (int)bi;
	}
	pdl_launch_dependents();
}

} // namespace cgpu
