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
#include "rowops.cuh"

namespace cgpu {

// The host expf table covers |x| in [2^-26, 2^7): biased exponents 101..133,
// both signs, every mantissa. Below it expf rounds to 1; at and above 128 it
// is +inf (x > 0) or 0 (x < 0).
constexpr uint32_t EXPTAB_E0 = 101, EXPTAB_NE = 33;
constexpr uint64_t EXPTAB_ENTRIES = 2ull * EXPTAB_NE << 23;

// The step's small device inputs and outputs: the token, its position, the
// argmax of its logits, the argmax's arrival ticket (zero between steps), and
// the index of the next token a device-side greedy run writes.
constexpr int FWD_IO_TOKEN = 0, FWD_IO_POS = 1, FWD_IO_NEXT = 2, FWD_IO_TICKET = 3,
	      FWD_IO_STEP = 4, FWD_IO_WORDS = 5;

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

// The test hook's kernel, one CTA of ORDERED_SUM_THREADS: out[0] =
// ordered_sum_seq(a[0..n)) and out[1] = ordered_sum_nonneg_cta of the same,
// from shared memory.
constexpr uint32_t ORDERED_SUM_MAX_N = 8192;
constexpr int ORDERED_SUM_THREADS = 512;

__global__ void __launch_bounds__(ORDERED_SUM_THREADS)
ordered_sum_kernel(const float *__restrict__ a, uint32_t n, float *__restrict__ out)
{
	__shared__ __align__(16) float sm[ORDERED_SUM_MAX_N];
	__shared__ OsumShared osum;
	for (uint32_t i = threadIdx.x; i < n; i += blockDim.x)
		sm[i] = a[i];
	__syncthreads();
	if (threadIdx.x == 0)
		out[0] = ordered_sum_seq(sm, n);
	const float s = n <= 4 * blockDim.x ? ordered_sum_nonneg_cta<4>(sm, n, osum)
					    : ordered_sum_nonneg_cta<16>(sm, n, osum);
	if (threadIdx.x == 0)
		out[1] = s;
}

// x (+ add, written back to x when add is given), then rmsnorm with weights
// w (src/llama.c:316-326: ss += x*x in order, scale = 1 / sqrtf(ss / n + eps),
// out = x * scale * w), then the quantiser of the result. One CTA; n a
// multiple of 32, at most FWD_NORM_MAX. The weights are fetched before the
// previous kernel is done (they do not depend on it), the squares by every
// thread, their ordered sum by the CTA (ordered_sum_nonneg_cta).
constexpr uint32_t FWD_NORM_MAX = 8192;
constexpr int FWD_NORM_THREADS = 512;

inline size_t fwd_norm_smem(uint32_t n)
{
	return (size_t)3 * n * sizeof(float);
}

__global__ void __launch_bounds__(FWD_NORM_THREADS)
fwd_norm_quant_kernel(float *__restrict__ x, const float *__restrict__ add,
		      const float *__restrict__ w, uint32_t n, float eps, int8_t *__restrict__ q,
		      float *__restrict__ d)
{
	extern __shared__ __align__(16) float nsm[];
	float *xs = nsm, *sq = nsm + n, *ws = nsm + 2 * n;      // fwd_norm_smem(n)
	__shared__ float scale_s;
	for (uint32_t i = threadIdx.x * 4; i < n; i += blockDim.x * 4)
		cp_async16(ws + i, w + i);
	pdl_wait();
	// the next kernel (a matvec) may launch now and start its weight loads
	// while the chain runs; it reads nothing of this one's before its own
	// wait, which returns once this grid is done
	pdl_launch_dependents();
	norm_quant_cta(x, add, n, eps, xs, sq, ws, &scale_s, q, d);
	if (add)
		for (uint32_t i = threadIdx.x; i < n; i += blockDim.x)
			x[i] = xs[i];
}

// The same rmsnorm in charsiu's NPU number format: the result quantised with
// one scale for the whole vector (quantise_one_cta) into q1 (kp bytes) and
// *d1, for the NPU-format matvec after it (src/llama.c:255-290).
__global__ void __launch_bounds__(FWD_NORM_THREADS)
fwd_norm_q1_kernel(float *__restrict__ x, const float *__restrict__ add,
		   const float *__restrict__ w, uint32_t n, float eps, uint32_t kp,
		   int8_t *__restrict__ q1, float *__restrict__ d1)
{
	extern __shared__ __align__(16) float nsm[];
	float *xs = nsm, *sq = nsm + n, *ws = nsm + 2 * n;      // fwd_norm_smem(n)
	__shared__ float scale_s, red[32];
	for (uint32_t i = threadIdx.x * 4; i < n; i += blockDim.x * 4)
		cp_async16(ws + i, w + i);
	pdl_wait();
	pdl_launch_dependents();
	const float scale = norm_scale_cta(x, add, n, eps, xs, sq, &scale_s);
	quantise_one_cta([&](uint32_t i) { return __fmul_rn(__fmul_rn(xs[i], scale), ws[i]); }, n,
			 kp, q1, d1, red);
	if (add)
		for (uint32_t i = threadIdx.x; i < n; i += blockDim.x)
			x[i] = xs[i];
}

// The NPU number format's activation of an fp32 vector (the attention output
// before the o projection, SiLU's before down): one CTA, the n values staged
// in shared memory, then quantise_one_cta into q1 (kp bytes) and *d1.
constexpr int FWD_Q1_THREADS = 1024;

__global__ void __launch_bounds__(FWD_Q1_THREADS)
fwd_q1_kernel(const float *__restrict__ v, uint32_t n, uint32_t kp, int8_t *__restrict__ q1,
	      float *__restrict__ d1)
{
	extern __shared__ __align__(16) float vsm[];            // n floats
	__shared__ float red[32];
	pdl_wait();
	pdl_launch_dependents();
	for (uint32_t i = threadIdx.x; i < n; i += blockDim.x)
		vsm[i] = v[i];
	__syncthreads();
	quantise_one_cta([&](uint32_t i) { return vsm[i]; }, n, kp, q1, d1, red);
}

// One head of attention at this token's position, RoPE and the KV cache
// included (src/llama.c:364-383, 781-817):
//   q and this head's k rotated by the position's (cos, sin) pairs, from a
//   table the host filled with the reference's own libm calls; the CTA of the
//   first query head of each KV head writes the rotated k and v into the
//   layer's cache row of the position (the other heads of the group rotate k
//   for themselves, the same bits, and read only rows before the position);
//   scores a_t = (sum_i q_i k_ti, in order) * scale; softmax (the max, expf,
//   the sum over t in order, the division); out_i = sum_t att_t v_ti in order
//   from 0; then the quantiser of the head's outputs (head_dim a multiple of
//   32, so every 32-block of the attention output lies inside one head), or,
//   when out_f is given, the outputs themselves into out_f[h * hd ..] (the NPU
//   number format quantises the whole vector at once, after this kernel).
// One CTA a head. K and V pass through shared memory a tile of positions at a
// time (rows of hd + 4 floats: 16-byte copies, and a float4 read a row per
// lane meets no bank conflict); the first tile's cache rows -- written by
// earlier tokens, so independent of the kernels before this one -- are
// copied in before this kernel waits on them. Each score's dot runs in one
// thread, the softmax sum in thread 0, each out_i in one thread.
constexpr int FWD_ATTN_THREADS = 256;
constexpr size_t FWD_ATTN_TILE_BYTES = 140 * 1024;      // both tiles

inline uint32_t fwd_attention_tile(uint32_t hd)
{
	uint32_t t = (uint32_t)(FWD_ATTN_TILE_BYTES / (2 * (hd + 4) * sizeof(float)));
	t = t > (uint32_t)FWD_ATTN_THREADS ? (uint32_t)FWD_ATTN_THREADS : t;
	return t / 32 * 32;
}

// the scores' region, rounded up to whole 16-byte words so the tiles after it
// start on a 16-byte boundary (their float4 reads and 16-byte copies need one)
__host__ __device__ inline uint32_t fwd_attention_att_floats(uint32_t n_ctx)
{
	return (n_ctx + 3u) & ~3u;
}

inline size_t fwd_attention_smem(uint32_t n_ctx, uint32_t hd)
{
	return ((size_t)fwd_attention_att_floats(n_ctx) + 4 * hd +
		2 * (size_t)fwd_attention_tile(hd) * (hd + 4)) * sizeof(float);
}

// One head h of the attention above, by the threads of G: fsm is the dynamic
// shared memory (fwd_attention_smem bytes), red 32 floats and *sum_sh one of
// shared memory. `wait` runs once the first tile's cache rows are on their
// way and before anything of this token's is read (the wait on the kernel or
// stage before).
template <class G, class Wait>
__device__ __forceinline__ void
attention_head(uint32_t h, float *fsm, float *red, float *sum_sh, Wait wait,
	       const float *__restrict__ qv, const float *__restrict__ kv,
	       const float *__restrict__ vv, const float *__restrict__ rope_cs,
	       float *__restrict__ kcache, float *__restrict__ vcache, const int *__restrict__ io,
	       uint32_t n_head, uint32_t n_head_kv, uint32_t hd, uint32_t n_ctx, uint32_t tile,
	       float scale, const float *__restrict__ exptab, int8_t *__restrict__ q,
	       float *__restrict__ d, float *__restrict__ out_f)
{
	const uint32_t tid = G::tid(), nthr = G::size();
	const uint32_t rs = hd + 4;
	float *att = fsm;                  // n_ctx scores
	float *qs = att + fwd_attention_att_floats(n_ctx);     // this head's q, rotated
	float *kp = qs + hd;               // its KV head's k at this position, rotated
	float *vp = kp + hd;               // and v
	float *os = vp + hd;               // this head's outputs
	float *kt = os + hd;               // tile rows of K
	float *vt = kt + (size_t)tile * rs;
	const uint32_t kvdim = n_head_kv * hd, gqa = n_head / n_head_kv;
	const uint32_t kvh = h / gqa;
	// the position came in with the step's first copy, before any kernel of it
	const int pos = io[FWD_IO_POS], np = pos + 1;
	float *kc = kcache + kvh * hd, *vc = vcache + kvh * hd;
	// cache rows t0 .. t0 + nt - 1 below pos into a tile
	auto issue = [&](float *dst, const float *cache, int t0, int nt) {
		const uint32_t q4 = hd / 4;
		for (uint32_t j = tid; j < (uint32_t)nt * q4; j += nthr) {
			const int t = t0 + (int)(j / q4);
			const uint32_t i = (j % q4) * 4;
			if (t < pos)
				cp_async16(dst + (size_t)(t - t0) * rs + i, cache + (size_t)t * kvdim + i);
		}
	};
	// and row pos, when the tile holds it, from this head's own copy
	auto own_row = [&](float *dst, const float *own, int t0, int nt) {
		if (pos >= t0 && pos < t0 + nt)
			for (uint32_t i = tid; i < hd; i += nthr)
				dst[(size_t)(pos - t0) * rs + i] = own[i];
	};
	const int nt0 = np < (int)tile ? np : (int)tile;
	issue(kt, kc, 0, nt0);
	issue(vt, vc, 0, nt0);
	wait();
	const float *cs = rope_cs + (size_t)pos * hd;
	for (uint32_t i = tid; i < hd / 2; i += nthr) {
		const float c = cs[2 * i], s = cs[2 * i + 1];
		float x0 = qv[h * hd + 2 * i], x1 = qv[h * hd + 2 * i + 1];
		qs[2 * i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
		qs[2 * i + 1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
		x0 = kv[kvh * hd + 2 * i];
		x1 = kv[kvh * hd + 2 * i + 1];
		kp[2 * i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
		kp[2 * i + 1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
	}
	for (uint32_t i = tid; i < hd; i += nthr)
		vp[i] = vv[kvh * hd + i];
	G::sync();
	if (h % gqa == 0)
		for (uint32_t i = tid; i < hd; i += nthr) {
			kc[(size_t)pos * kvdim + i] = kp[i];
			vc[(size_t)pos * kvdim + i] = vp[i];
		}
	own_row(kt, kp, 0, nt0);
	own_row(vt, vp, 0, nt0);
	cp_async_wait_all();
	G::sync();
	for (int t0 = 0; t0 < np; t0 += (int)tile) {
		const int nt = np - t0 < (int)tile ? np - t0 : (int)tile;
		if (t0) {
			G::sync();
			issue(kt, kc, t0, nt);
			own_row(kt, kp, t0, nt);
			cp_async_wait_all();
			G::sync();
		}
		if ((int)tid < nt) {
			const float4 *k4 = reinterpret_cast<const float4 *>(kt + (size_t)tid * rs);
			float a = 0.0f;
			for (uint32_t i = 0; i < hd / 4; i++) {
				const float4 k = k4[i];
				a = __fadd_rn(a, __fmul_rn(qs[4 * i], k.x));
				a = __fadd_rn(a, __fmul_rn(qs[4 * i + 1], k.y));
				a = __fadd_rn(a, __fmul_rn(qs[4 * i + 2], k.z));
				a = __fadd_rn(a, __fmul_rn(qs[4 * i + 3], k.w));
			}
			att[t0 + tid] = __fmul_rn(a, scale);
		}
	}
	G::sync();
	// the max: any order gives the reference's value for NaN-free scores (a NaN
	// needs a non-finite weight or delta)
	float mx = -__int_as_float(0x7f800000);
	for (int t = tid; t < np; t += nthr)
		mx = fmaxf(mx, att[t]);
	for (int o = 16; o; o >>= 1)
		mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
	if ((tid & 31) == 0)
		red[tid >> 5] = mx;
	G::sync();
	mx = red[0];
	for (uint32_t wi = 1; wi < nthr / 32; wi++)
		mx = fmaxf(mx, red[wi]);
	for (int t = tid; t < np; t += nthr)
		att[t] = exp_exact(__fsub_rn(att[t], mx), exptab);
	G::sync();
	if (tid == 0)
		*sum_sh = ordered_sum_seq(att, (uint32_t)np);
	G::sync();
	const float sum = *sum_sh;
	for (int t = tid; t < np; t += nthr)
		att[t] = __fdiv_rn(att[t], sum);
	G::sync();
	float o = 0.0f;
	for (int t0 = 0; t0 < np; t0 += (int)tile) {
		const int nt = np - t0 < (int)tile ? np - t0 : (int)tile;
		if (t0) {
			G::sync();
			issue(vt, vc, t0, nt);
			own_row(vt, vp, t0, nt);
			cp_async_wait_all();
			G::sync();
		}
		if (tid < hd)
#pragma unroll 4
			for (int t = 0; t < nt; t++)
				o = __fadd_rn(o, __fmul_rn(att[t0 + t], vt[(size_t)t * rs + tid]));
	}
	if (out_f) {
		if (tid < hd)
			out_f[h * hd + tid] = o;
		return;
	}
	if (tid < hd)
		os[tid] = o;
	G::sync();
	const int warp = tid >> 5, lane = tid & 31;
	for (uint32_t b = warp; b < hd / 32; b += nthr / 32) {
		const uint32_t e = h * hd + b * 32;
		quantise_block_warp(os[b * 32 + lane], lane, q + e, d + e / 32);
	}
}

__global__ void __launch_bounds__(FWD_ATTN_THREADS)
fwd_attention_kernel(const float *__restrict__ qv, const float *__restrict__ kv,
		     const float *__restrict__ vv, const float *__restrict__ rope_cs,
		     float *__restrict__ kcache, float *__restrict__ vcache,
		     const int *__restrict__ io, uint32_t n_head, uint32_t n_head_kv, uint32_t hd,
		     uint32_t n_ctx, uint32_t tile, float scale, const float *__restrict__ exptab,
		     int8_t *__restrict__ q, float *__restrict__ d, float *__restrict__ out_f)
{
	extern __shared__ __align__(16) float fsm[];
	__shared__ float red[32];
	__shared__ float sum_s;
	attention_head<CtaGroup>(blockIdx.x, fsm, red, &sum_s,
				 [] { pdl_wait(); pdl_launch_dependents(); }, qv, kv, vv, rope_cs,
				 kcache, vcache, io, n_head, n_head_kv, hd, n_ctx, tile, scale, exptab,
				 q, d, out_f);
}

// SiLU(gate) * up (src/llama.c:831-836: g *= 1 / (1 + expf(-g)); g * up),
// then the quantiser of the result, one warp a 32-block -- or, when out_f is
// given, the result itself into out_f (the NPU number format's path).
__global__ void fwd_silu_quant_kernel(const float *__restrict__ gate, const float *__restrict__ up,
				      uint32_t n, const float *__restrict__ exptab,
				      int8_t *__restrict__ q, float *__restrict__ d,
				      float *__restrict__ out_f)
{
	pdl_wait();
	pdl_launch_dependents();
	const uint32_t b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
	const int lane = threadIdx.x & 31;
	if (b < n / 32) {
		const uint32_t i = b * 32 + lane;
		float g = gate[i];
		const float e = exp_exact(-g, exptab);
		g = __fmul_rn(g, __fdiv_rn(1.0f, __fadd_rn(1.0f, e)));
		if (out_f)
			out_f[i] = __fmul_rn(g, up[i]);
		else
			quantise_block_warp(__fmul_rn(g, up[i]), lane, q + b * 32, d + b);
	}
}

// llama_argmax (src/llama.c:860-868): the first index of the maximum, a NaN
// never taken past index 0 (and index 0 kept when it is NaN), into
// io[FWD_IO_NEXT]. Each thread keeps the first maximum of the elements it
// visits (in increasing index order); (value, index) pairs then merge by the
// larger value, the smaller index on a tie, over the warp, the CTA, and --
// in the CTA that arrives last on `ticket` -- the grid's per-CTA results
// (`part`, FWD_ARGMAX_CTAS pairs). The last CTA resets the ticket.
constexpr int FWD_ARGMAX_THREADS = 256, FWD_ARGMAX_CTAS = 64;
constexpr uint32_t ARGMAX_NONE = 0xffffffffu;

__device__ __forceinline__ void argmax_merge(float &bv, uint32_t &bi, float ov, uint32_t oi)
{
	if (oi != ARGMAX_NONE && (bi == ARGMAX_NONE || ov > bv || (ov == bv && oi < bi))) {
		bv = ov;
		bi = oi;
	}
}

__device__ __forceinline__ void argmax_block(float &bv, uint32_t &bi, float *rv, uint32_t *ri)
{
	for (int o = 16; o; o >>= 1) {
		const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
		const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
		argmax_merge(bv, bi, ov, oi);
	}
	if ((threadIdx.x & 31) == 0) {
		rv[threadIdx.x >> 5] = bv;
		ri[threadIdx.x >> 5] = bi;
	}
	__syncthreads();
	if (threadIdx.x == 0)
		for (int w = 1; w < (int)(blockDim.x / 32); w++)
			argmax_merge(bv, bi, rv[w], ri[w]);
}

__global__ void __launch_bounds__(FWD_ARGMAX_THREADS)
fwd_argmax_kernel(const float *__restrict__ x, uint32_t n, int *__restrict__ io,
		  uint32_t *__restrict__ ticket, float *__restrict__ part_v,
		  uint32_t *__restrict__ part_i)
{
	__shared__ float rv[FWD_ARGMAX_THREADS / 32];
	__shared__ uint32_t ri[FWD_ARGMAX_THREADS / 32];
	pdl_wait();
	pdl_launch_dependents();
	float bv = -__int_as_float(0x7f800000);
	uint32_t bi = ARGMAX_NONE;
	auto take = [&](float v, uint32_t i) {
		if (v > bv || (v == bv && bi == ARGMAX_NONE)) {
			bv = v;
			bi = i;
		}
	};
	const float4 *x4 = reinterpret_cast<const float4 *>(x);
	const uint32_t n4 = n / 4, stride = gridDim.x * blockDim.x;
	for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < n4; j += stride) {
		const float4 v = x4[j];
		take(v.x, 4 * j);
		take(v.y, 4 * j + 1);
		take(v.z, 4 * j + 2);
		take(v.w, 4 * j + 3);
	}
	if (blockIdx.x == 0 && threadIdx.x < n - n4 * 4)
		take(x[n4 * 4 + threadIdx.x], n4 * 4 + threadIdx.x);
	argmax_block(bv, bi, rv, ri);
	if (threadIdx.x == 0) {
		part_v[blockIdx.x] = bv;
		part_i[blockIdx.x] = bi;
		if (atom_add_acq_rel_gpu(ticket, 1u) == gridDim.x - 1) {
			*ticket = 0;
			float fv = part_v[0];
			uint32_t fi = part_i[0];
			for (uint32_t c = 1; c < gridDim.x; c++)
				argmax_merge(fv, fi, ((volatile float *)part_v)[c],
					     ((volatile uint32_t *)part_i)[c]);
			const float x0 = x[0];
			io[FWD_IO_NEXT] = (x0 != x0 || fi == ARGMAX_NONE) ? 0 : (int)fi;
		}
	}
}

// The greedy loop's step on the device (tools/charsiu_run.c:295-317 without
// the host): the argmax just taken becomes the next step's token, at the next
// position, and is appended to out. The host checked that every position the
// run reaches is inside the context, so the caches are never indexed past it.
__global__ void fwd_advance_kernel(int *__restrict__ io, int32_t *__restrict__ out)
{
	pdl_wait();
	if (threadIdx.x == 0) {
		const int next = io[FWD_IO_NEXT];
		out[io[FWD_IO_STEP]] = next;
		io[FWD_IO_STEP] += 1;
		io[FWD_IO_TOKEN] = next;
		io[FWD_IO_POS] += 1;
	}
}

} // namespace cgpu
