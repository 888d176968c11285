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

// The threads a row operation runs on: the whole CTA (the decode step's own
// kernels), or NW warps from warp W0 on, synchronised by named barrier BAR
// (the persistent step kernel, whose other warps stream weights meanwhile).
struct CtaGroup {
	__device__ static uint32_t tid() { return threadIdx.x; }
	__device__ static uint32_t size() { return blockDim.x; }
	__device__ static void sync() { __syncthreads(); }
};

template <int W0, int NW, int BAR>
struct WarpGroup {
	__device__ static uint32_t tid() { return threadIdx.x - W0 * 32; }
	__device__ static constexpr uint32_t size() { return NW * 32; }
	__device__ static void sync()
	{
		asm volatile("bar.sync %0, %1;" :: "n"(BAR), "n"(NW * 32) : "memory");
	}
};

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

// The same sum, bit for bit, by a whole CTA, for terms that are all >= +0
// and finite (the rmsnorm's squares); any other term sends the CTA down
// ordered_sum_seq. Exact, not approximate: while the running sum s stays in
// one binade [2^e, 2^(e+1)) it is m * u on that binade's grid
// (u = 2^(e-23), m an integer in [2^23, 2^24)), and adding a term t that
// keeps it there rounds (m + t/u) to the nearest integer, ties to even. So
// away from binade changes and ties the sum is an integer prefix sum of
// q = rne(t/u), which one CTA scan computes for all terms at once:
//  1. an fp32 prefix sum of the terms (any order) predicts the binade of the
//     running sum before each term; a term after which the prediction
//     changes binade (and the last term) is a CROSSING;
//  2. per term q = rne(t/u) on its predicted grid (ties: rounded down and
//     flagged), and one 64-bit exclusive scan of q | ties << 40 | crossings
//     << 52 gives every term its grid offset and its rank among the ties
//     and crossings, which list themselves in shared memory;
//  3. warp 0 walks the crossings in order. Each lane first prepares one or
//     two crossings in parallel: the run of grid terms before it, its offset,
//     and how many of its ties round up (a tie rounds up when m + floor(t/u)
//     is odd at that point) for either parity of m at the run's start. Then,
//     crossing by crossing, in registers: check that s is in the predicted
//     binade, add the run's offset and round-ups to m, check that m stayed
//     below 2^24, and add the crossing term with a real fp32 add.
// A failed check (the fp32 prediction off near a power of two, too many
// ties or crossings to list) makes lane 0 finish with plain adds from the
// last exact point, so the result is always the sequential sum. Terms are
// read EPT a thread at most (n <= EPT * blockDim, else the sequential form);
// every thread gets the sum.
constexpr int OSUM_CMAX = 64;       // crossings listed
constexpr int OSUM_TMAX = 256;      // ties listed

struct OsumShared {
	float wf[32];                    // per-warp fp32 totals
	unsigned long long wq[32];       // per-warp packed totals
	uint32_t wbad[32];               // per-warp: a term that is not >= +0 and finite
	uint32_t c_idx[OSUM_CMAX], c_qx[OSUM_CMAX], c_b[OSUM_CMAX], c_t[OSUM_CMAX];
	uint32_t t_qx[OSUM_TMAX], t_k[OSUM_TMAX];
	float result;
};

__device__ __forceinline__ uint32_t binade_field(float v)
{
	return (__float_as_uint(v) >> 23) & 0xffu;
}

template <int EPT, class G = CtaGroup>
__device__ float ordered_sum_nonneg_cta(const float *t, uint32_t n, OsumShared &sh)
{
	const uint32_t tid = G::tid(), nt = G::size(), lane = tid & 31, wid = tid >> 5;
	const uint32_t ept = (n + nt - 1) / nt;
	const uint32_t i0 = tid * ept;
	float v[EPT];
	bool bad = ept > (uint32_t)EPT;
#pragma unroll
	for (int k = 0; k < EPT; k++) {
		const uint32_t i = i0 + k;
		v[k] = ((uint32_t)k < ept && i < n) ? t[i] : 0.0f;
		bad |= !(v[k] >= 0.0f && v[k] <= 3.402823466e38f);       // NaN, < 0, inf
	}

	// 1. fp32 prefix sums (this thread's terms in order, then warps, then the
	//    CTA), only to predict binades
	float tsum = 0.0f;
#pragma unroll
	for (int k = 0; k < EPT; k++)
		tsum = __fadd_rn(tsum, v[k]);
	float inc = tsum;
#pragma unroll
	for (int o = 1; o < 32; o <<= 1) {
		const float y = __shfl_up_sync(0xffffffffu, inc, o);
		if (lane >= (uint32_t)o)
			inc = __fadd_rn(inc, y);
	}
	float ex = __shfl_up_sync(0xffffffffu, inc, 1);
	if (lane == 0)
		ex = 0.0f;
	bad = __any_sync(0xffffffffu, bad);
	if (lane == 31) {
		sh.wf[wid] = inc;
		sh.wbad[wid] = bad;
	}
	G::sync();
	// every warp turns the warp totals into the warps' starting values itself
	// (the same operations on the same values in every warp, so the same bits:
	// warp w starts at woff(w), which the last lane of warp w - 1 also uses)
	const uint32_t nw = nt / 32;
	float woff_in;                          // lane l: the sum of warps 0..l
	{
		const float y = lane < nw ? sh.wf[lane] : 0.0f;
		bad = __any_sync(0xffffffffu, lane < nw && sh.wbad[lane]);
		woff_in = y;
#pragma unroll
		for (int o = 1; o < 32; o <<= 1) {
			const float z = __shfl_up_sync(0xffffffffu, woff_in, o);
			if (lane >= (uint32_t)o)
				woff_in = __fadd_rn(woff_in, z);
		}
	}
	if (bad) {
		if (tid == 0)
			sh.result = ordered_sum_seq(t, n);
		G::sync();
		return sh.result;
	}
	const float w_start = wid ? __shfl_sync(0xffffffffu, woff_in, wid - 1) : 0.0f;
	const float w_next = __shfl_sync(0xffffffffu, woff_in, wid);
	float X = __fadd_rn(w_start, ex);
	// the prediction after this thread's last term must be the very value the
	// next thread starts from (its X), so that the runs of step 3 never mix
	// two predicted grids: the next lane's X, or the next warp's first
	float x_next = __shfl_down_sync(0xffffffffu, X, 1);
	if (lane == 31)
		x_next = w_next;

	// 2. grid offsets, ties, crossings
	unsigned long long pk[EPT];
	uint32_t bk[EPT];
	unsigned long long lsum = 0;
#pragma unroll
	for (int k = 0; k < EPT; k++) {
		const uint32_t i = i0 + k;
		const float P = (uint32_t)k + 1 == ept ? x_next : __fadd_rn(X, v[k]);
		const uint32_t b = binade_field(X), bn = binade_field(P);
		bk[k] = b;
		unsigned long long q = 1ull << 52;                      // a crossing
		if (b == bn && b >= 23 && b <= 254 && i != n - 1) {
			const float f = __fmul_rn(v[k], __uint_as_float((277u - b) << 23));  // t / u
			if (f < 4194304.0f) {
				// rne(f) by adding 1.5 * 2^23 (exact below 2^22); a tie is
				// a rounding by exactly one half, taken down here
				const float g = __fadd_rn(f, 12582912.0f);
				const uint32_t r = __float_as_uint(g) - 0x4b400000u;
				const float dr = __fsub_rn(__fsub_rn(g, 12582912.0f), f);
				const bool tie = fabsf(dr) == 0.5f;
				q = tie ? ((unsigned long long)(r - (dr > 0.0f)) | 1ull << 40)
					: (unsigned long long)r;
			}
		}
		pk[k] = ((uint32_t)k < ept && i < n) ? q : 0ull;
		lsum += pk[k];
		X = P;
	}
	unsigned long long qinc = lsum;
#pragma unroll
	for (int o = 1; o < 32; o <<= 1) {
		const unsigned long long y = __shfl_up_sync(0xffffffffu, qinc, o);
		if (lane >= (uint32_t)o)
			qinc += y;
	}
	unsigned long long qex = qinc - lsum;
	if (lane == 31)
		sh.wq[wid] = qinc;
	G::sync();
	// (again every warp scans the warp totals itself)
	unsigned long long q_all;
	{
		const unsigned long long y = lane < nw ? sh.wq[lane] : 0ull;
		unsigned long long wi = y;
#pragma unroll
		for (int o = 1; o < 32; o <<= 1) {
			const unsigned long long z = __shfl_up_sync(0xffffffffu, wi, o);
			if (lane >= (uint32_t)o)
				wi += z;
		}
		qex += __shfl_sync(0xffffffffu, wi - y, wid);
		q_all = __shfl_sync(0xffffffffu, wi, 31);
	}
	// (only the few threads holding a tie or a crossing list anything)
#pragma unroll
	for (int k = 0; k < EPT; k++) {
		if (!(lsum >> 40))
			break;
		const uint32_t i = i0 + k;
		if (pk[k] >> 52) {
			const uint32_t r = (uint32_t)(qex >> 52);
			if (r < OSUM_CMAX) {
				sh.c_idx[r] = i;
				sh.c_qx[r] = (uint32_t)qex;
				sh.c_b[r] = bk[k];
				sh.c_t[r] = (uint32_t)(qex >> 40) & 0xfffu;     // ties before it
			}
		} else if ((pk[k] >> 40) & 0xfffu) {
			const uint32_t r = (uint32_t)(qex >> 40) & 0xfffu;
			if (r < OSUM_TMAX) {
				sh.t_qx[r] = (uint32_t)qex;
				sh.t_k[r] = (uint32_t)pk[k];
			}
		}
		qex += pk[k];
	}
	G::sync();

	// 3. warp 0: each lane prepares crossings lane and lane + 32 -- the run of
	//    grid terms before it (its offset, and what its ties add for either
	//    parity of m at the run's start), then the chain over the crossings
	//    in order, in registers
	if (wid == 0) {
		const uint32_t nc = (uint32_t)(q_all >> 52), ntie = (uint32_t)(q_all >> 40) & 0xfffu;
		bool ok = nc <= (uint32_t)OSUM_CMAX && ntie <= (uint32_t)OSUM_TMAX;
		// per crossing: the term, the run's offset, and a word of the
		// predicted binade (bits 0..7), whether a run precedes it (bit 8) and
		// its ties' round-ups for m even (bits 9..17) and odd (18..26)
		float tc[2];
		uint32_t rq[2], rw[2];
#pragma unroll
		for (int h = 0; h < 2; h++) {
			const uint32_t r = lane + 32 * h;
			tc[h] = 0.0f;
			rq[h] = rw[h] = 0;
			if (ok && r < nc) {
				const uint32_t c = sh.c_idx[r], st = r ? sh.c_idx[r - 1] + 1 : 0;
				const uint32_t q0 = r ? sh.c_qx[r - 1] : 0, t0 = r ? sh.c_t[r - 1] : 0;
				tc[h] = t[c];
				rq[h] = sh.c_qx[r] - q0;
				uint32_t up0 = 0, up1 = 0;
				for (uint32_t j = t0; j < sh.c_t[r]; j++) {
					const uint32_t o = sh.t_qx[j] - q0 + sh.t_k[j];
					up0 += (o + up0) & 1u;
					up1 += (1u + o + up1) & 1u;
				}
				rw[h] = sh.c_b[r] | (c > st ? 1u << 8 : 0u) | up0 << 9 | up1 << 18;
			}
		}
		// batches of 8 crossings: all of a batch's shuffles first, then the
		// chain through them in registers
		float s = 0.0f;
		uint32_t done = 0;
		for (uint32_t r0 = 0; ok && r0 < nc; r0 += 8) {
			float bt[8];
			uint32_t bq[8], bw[8];
			const int h = (r0 >> 5) & 1;        // r0 + 7 stays in the same half
#pragma unroll
			for (int j = 0; j < 8; j++) {
				const int src = (r0 + j) & 31;
				bt[j] = __shfl_sync(0xffffffffu, h ? tc[1] : tc[0], src);
				bq[j] = __shfl_sync(0xffffffffu, h ? rq[1] : rq[0], src);
				bw[j] = __shfl_sync(0xffffffffu, h ? rw[1] : rw[0], src);
			}
#pragma unroll
			for (int j = 0; j < 8; j++) {
				// (selects, no branches: the chain is the step's latency)
				const uint32_t w = bw[j], b = w & 0xffu;
				const bool run = w & (1u << 8), live = r0 + j < nc;
				const uint32_t m = (__float_as_uint(s) & 0x7fffffu) | 0x800000u;
				const uint32_t mend =
					m + bq[j] + ((m & 1u) ? w >> 18 : (w >> 9) & 0x1ffu);
				const bool bad = run && (binade_field(s) != b || mend >= 0x1000000u);
				const float sg = run ? __uint_as_float((b << 23) | (mend & 0x7fffffu)) : s;
				const float sn = __fadd_rn(sg, bt[j]);
				const bool take = ok && live && !bad;
				s = take ? sn : s;
				done = take ? r0 + j + 1 : done;
				ok = ok && !(live && bad);
			}
		}
		if (lane == 0) {
			if (!ok)
				for (uint32_t i = done ? sh.c_idx[done - 1] + 1 : 0; i < n; i++)
					s = __fadd_rn(s, t[i]);
			sh.result = s;
		}
	}
	G::sync();
	return sh.result;
}

// rmsnorm's scale (reference src/llama.c:316-326) of x (+ add), by the whole
// CTA: xs[i] = x[i] + add[i] (x alone when add is null), ss = the ordered sum
// of xs[i]^2 (the CTA's exact form, ordered_sum_nonneg_cta), and the returned
// scale = 1 / sqrtf(ss / n + eps) (through *scale_sh, a shared float). xs, sq:
// n floats each of shared memory, 16-byte aligned. Ends with a barrier.
template <class G = CtaGroup>
__device__ __forceinline__ float norm_scale_cta(const float *__restrict__ x,
						const float *__restrict__ add, uint32_t n,
						float eps, float *xs, float *sq, float *scale_sh)
{
	for (uint32_t i = G::tid(); i < n; i += G::size()) {
		float v = x[i];
		if (add)
			v = __fadd_rn(v, add[i]);
		xs[i] = v;
		sq[i] = __fmul_rn(v, v);
	}
	cp_async_wait_all();
	G::sync();
	__shared__ OsumShared osum;
	const float ss = n <= 4 * G::size() ? ordered_sum_nonneg_cta<4, G>(sq, n, osum)
					    : ordered_sum_nonneg_cta<16, G>(sq, n, osum);
	if (G::tid() == 0)
		*scale_sh = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
	G::sync();
	return *scale_sh;
}

// charsiu_act_set's single-scale form (src/gguf.c:883-910), the NPU number
// format's activation, of n values by the whole CTA: d1 = amax / 127 (a max,
// so any order), q1[i] = lrintf(v_i * (1 / d1)) clamped to [-127, 127], zero
// from n to kp. val(i) gives v_i (called twice per element); red: 32 floats
// of shared memory. Ends with a barrier.
template <class V>
__device__ __forceinline__ void quantise_one_cta(V val, uint32_t n, uint32_t kp, int8_t *q1,
						 float *d1, float *red)
{
	const uint32_t tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, wid = tid >> 5;
	float amax = 0.0f;
	for (uint32_t i = tid; i < n; i += nt)
		amax = fmaxf(amax, fabsf(val(i)));
	for (int o = 16; o; o >>= 1)
		amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
	if (lane == 0)
		red[wid] = amax;
	__syncthreads();
	amax = 0.0f;
	for (uint32_t w = 0; w < nt / 32; w++)
		amax = fmaxf(amax, red[w]);
	const float d = __fdiv_rn(amax, 127.0f);
	const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
	if (tid == 0)
		*d1 = d;
	for (uint32_t i = tid; i < kp; i += nt) {
		int v = 0;
		if (i < n)
			v = min(max(__float2int_rn(__fmul_rn(val(i), id)), -127), 127);
		q1[i] = (int8_t)v;
	}
	__syncthreads();
}

// rmsnorm of x (+ add) as norm_scale_cta, then the quantiser of the result
// v = xs[i] * scale * w[i] into aq / ad, one warp a 32-block. ws: n floats
// of shared memory holding w already (copied in by the caller). Ends with a
// barrier; xs still holds x + add.
template <class G = CtaGroup>
__device__ __forceinline__ void norm_quant_cta(const float *__restrict__ x,
					       const float *__restrict__ add, uint32_t n, float eps,
					       float *xs, float *sq, const float *ws, float *scale_sh,
					       int8_t *aq, float *ad)
{
	const float scale = norm_scale_cta<G>(x, add, n, eps, xs, sq, scale_sh);
	const int warp = G::tid() >> 5, lane = G::tid() & 31;
	const uint32_t nw = G::size() / 32;
	uint32_t b = warp;
	// four blocks of a warp at a time, their reductions and divisions
	// interleaved (blocks b, b + nw, b + 2 nw, b + 3 nw)
	for (; b + 3 * nw < n / 32; b += 4 * nw) {
		float v[4], amax[4];
#pragma unroll
		for (int j = 0; j < 4; j++) {
			const uint32_t i = (b + j * nw) * 32 + lane;
			v[j] = __fmul_rn(__fmul_rn(xs[i], scale), ws[i]);
			amax[j] = fabsf(v[j]);
		}
#pragma unroll
		for (int o = 16; o; o >>= 1)
#pragma unroll
			for (int j = 0; j < 4; j++)
				amax[j] = fmaxf(amax[j], __shfl_xor_sync(0xffffffffu, amax[j], o));
#pragma unroll
		for (int j = 0; j < 4; j++) {
			const float dd = __fdiv_rn(amax[j], 127.0f);
			const float inv = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
			aq[(b + j * nw) * 32 + lane] = (int8_t)__float2int_rn(__fmul_rn(v[j], inv));
			if (lane == 0)
				ad[b + j * nw] = dd;
		}
	}
	for (; b < n / 32; b += nw) {
		const uint32_t i = b * 32 + lane;
		quantise_block_warp(__fmul_rn(__fmul_rn(xs[i], scale), ws[i]), lane, aq + b * 32,
				    ad + b);
	}
	G::sync();
}

} // namespace cgpu
