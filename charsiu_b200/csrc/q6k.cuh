// SPDX-License-Identifier: GPL-2.0-or-later
// The q6_K matvec (one activation): charsiu's dotq_q6_K (reference
// src/gguf.c:1109-1145, super-block of :449-454), bit for bit.
//
// llama.cpp writes token_embd -- and so the tied output head, the largest
// matmul of the model -- as q6_K even in a q4_0 file, so a q4_0 model runs its
// head through this kernel.
//
// A q6_K super-block is 256 weights in 210 bytes: ql[128], qh[64], int8
// scales[16], fp16 d. Half h (128 weights) takes ql[h*64 ..], qh[h*32 ..] and
// scales[h*8 ..]; its byte l (0..31) of qh and bytes l, l + 32 of ql make four
// 6-bit weights, run k = 0..3 of the half: the low nibble of ql[l] (k = 0) or
// ql[l + 32] (k = 1), the high nibbles (k = 2, 3), each with bits 2k, 2k + 1
// of qh[l] above it, minus 32. Every 16 weights (l in g*16 .. g*16+15) share
// one scale, scales[g + 2k] of the half; the reference's row sum adds, in the
// order (super-block, half, g, k), the terms ((d * scale) * d_a) * t with t
// the exact int32 dot of those 16 weights and the activation's 16 bytes.
//
// Device layout (repacked at add, 16-byte aligned): a row is its super-blocks'
// first 208 bytes (ql, qh, scales) back to back, then the fp16 d's, padded to
// 16 bytes.
//
// Organised as the q8_0 decode matvec (qmv1.cuh): 8-row groups dealt round
// robin over a persistent grid of small CTAs whose W warps split a group's
// super-blocks. Lane L of warp w takes row L/4, half (L/2)&1 and g = L&1 of
// super-block w + W*u (slot u of U; passes of W*U super-blocks) -- three
// 16-byte loads and the half's 8 scale bytes -- so one warp-load covers 64
// contiguous bytes of each of the 8 rows, and computes its four terms with
// dp4a (unsigned 6-bit weights, so the -32 comes off as 32 * sum(activation):
// each 16-byte run's activation sum is made once, while the activation is
// staged, and the staged halves are padded apart so the lanes reading them
// together hit different banks).
// The terms go to the row's line of a term buffer at the reference's position
// ((i*2 + h)*2 + g)*4 + k; after one barrier lanes 0..7 of warp 0 add their
// row's line in that order while the other warps load the next group. The
// first group's bytes are loaded before the wait on the previous kernel, and
// every CTA lets the next launch start as soon as it starts.
//
// Measured against the form it replaced (a warp taking 8 whole rows, each
// row's 8 super-blocks an item loaded two items ahead, 8-warp CTAs, no load
// before the wait), same bits: the 2048 -> 128256 head 66.2 -> 43.1 us
// (3.26 -> 5.0 TB/s), K=2048 N=8192 8.3 -> 4.9 us, K=4096 N=4096 11.1 ->
// 5.3 us, K=8192 N=2048 14.7 -> 6.05 us (four warps in four passes there
// measured 20.8 us, hence W by K). The run sums made at staging and the padded
// activation then took the head to 38.0 us, K=8192 N=2048 to 5.66 us; holding
// the 4-warp form to 64 registers (8 CTAs an SM instead of 7) lost on the head
// (41.5 us).
#pragma once

#include "layout.h"
#include "ptx.cuh"
#include "qmv1.cuh"

namespace cgpu {

// GGUF rows (210-byte super-blocks) -> the device layout; one thread a
// super-block. Load time only.
__global__ void q6k_repack_kernel(const uint8_t *__restrict__ src, uint32_t nsb, uint32_t nr,
				  uint8_t *__restrict__ dst)
{
	const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
	if (idx >= (uint64_t)nr * nsb)
		return;
	const uint64_t row = idx / nsb;
	const uint32_t i = (uint32_t)(idx % nsb);
	const uint8_t *s = src + idx * 210;
	uint8_t *d = dst + row * q6k_row_bytes(nsb);
	for (uint32_t b = 0; b < 208; b++)
		d[(uint64_t)i * 208 + b] = s[b];
	d[(uint64_t)nsb * 208 + 2 * i] = s[208];
	d[(uint64_t)nsb * 208 + 2 * i + 1] = s[209];
}

struct Q6kParams {
	const uint8_t *w;          // this GPU's rows in the device layout
	float *y;
	uint32_t rows, nsb;
	const int8_t *q;           // activation [nsb * 256]
	const float *d;            // activation deltas [nsb * 8]
};

// W warps a CTA, U super-blocks a warp a pass.
__host__ __device__ inline uint32_t q6k_tstride(uint32_t nsb)
{
	return nsb * 16 + 4;           // floats a row's line: its terms + 4 (banks, 16-byte rows)
}

// Shared memory: the activation's super-blocks at Q6K_ASB bytes each, half h
// at h * Q6K_AHALF (the two halves' words then fall in different banks for
// the lanes that read them together); each 16-byte run's byte sum as int32
// [i][h][g][k]; the activation deltas; two term buffers.
constexpr uint32_t Q6K_AHALF = 160, Q6K_ASB = 320;

inline size_t q6k_smem_bytes(uint32_t nsb)
{
	return (size_t)nsb * Q6K_ASB + (size_t)nsb * 16 * sizeof(int32_t) +
	       (size_t)nsb * 8 * sizeof(float) + (size_t)2 * RG * q6k_tstride(nsb) * sizeof(float);
}

template <int W, int U>
__global__ void __launch_bounds__(W * 32)
q6k_kernel(const __grid_constant__ Q6kParams p)
{
	extern __shared__ __align__(128) uint8_t smem[];
	const uint32_t nsb = p.nsb;
	uint8_t *aq = smem;
	int32_t *xsum = reinterpret_cast<int32_t *>(smem + (size_t)nsb * Q6K_ASB);
	float *ad = reinterpret_cast<float *>(xsum + (size_t)nsb * 16);
	float *terms = ad + (size_t)nsb * 8;
	const uint32_t ts = q6k_tstride(nsb);
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const uint32_t r = lane >> 2, h = (lane >> 1) & 1, g = lane & 1;
	const uint64_t rs = q6k_row_bytes(nsb);
	const uint32_t groups = (p.rows + RG - 1) / RG;
	constexpr uint32_t PASS = W * U;
	const uint32_t npass = (nsb + PASS - 1) / PASS;

	struct Regs {
		uint4 ql0, ql1, qh;
		uint2 sc;
		uint16_t d;
	};
	Regs R[U];
	auto load = [&](uint32_t G, uint32_t ps) {
		const uint32_t row = G * RG + r;
		const uint8_t *wr = p.w + (uint64_t)(row < p.rows ? row : 0) * rs;
#pragma unroll
		for (int u = 0; u < U; u++) {
			const uint32_t i = ps * PASS + (uint32_t)(u * W + warp);
			if (row < p.rows && i < nsb) {
				const uint8_t *sb = wr + (size_t)i * 208;
				R[u].ql0 = ldg_stream(sb + h * 64 + g * 16);
				R[u].ql1 = ldg_stream(sb + h * 64 + 32 + g * 16);
				R[u].qh = ldg_stream(sb + 128 + h * 32 + g * 16);
				R[u].sc = *reinterpret_cast<const uint2 *>(sb + 192 + h * 8);
				R[u].d = ldg_stream_u16(wr + (size_t)nsb * 208 + 2 * i);
			} else {
				R[u] = Regs{};
			}
		}
	};
	auto compute = [&](uint32_t ps, float *tb) {
#pragma unroll
		for (int u = 0; u < U; u++) {
			const uint32_t i = ps * PASS + (uint32_t)(u * W + warp);
			if (i >= nsb)
				continue;
			const Regs &Q = R[u];
			const float dd = half_bits_to_float(Q.d);
			const uint8_t *xq = aq + (size_t)i * Q6K_ASB + h * Q6K_AHALF + g * 16;
			const int4 xs4 = *reinterpret_cast<const int4 *>(xsum + (size_t)i * 16 + h * 8 + g * 4);
			const int xs[4] = {xs4.x, xs4.y, xs4.z, xs4.w};
			const float *xd = ad + (size_t)i * 8 + h * 4;
			const uint32_t ql0w[4] = {Q.ql0.x, Q.ql0.y, Q.ql0.z, Q.ql0.w};
			const uint32_t ql1w[4] = {Q.ql1.x, Q.ql1.y, Q.ql1.z, Q.ql1.w};
			const uint32_t qhw[4] = {Q.qh.x, Q.qh.y, Q.qh.z, Q.qh.w};
			float tv[4];
#pragma unroll
			for (int k = 0; k < 4; k++) {
				const uint4 xv = *reinterpret_cast<const uint4 *>(xq + k * 32);
				const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
				int t = 0;
#pragma unroll
				for (int wd = 0; wd < 4; wd++) {
					const uint32_t lo = (k & 1) ? ql1w[wd] : ql0w[wd];
					const uint32_t nib = (k & 2) ? (lo >> 4) & 0x0f0f0f0fu
								     : lo & 0x0f0f0f0fu;
					const uint32_t hi = (qhw[wd] >> (2 * k)) & 0x03030303u;
					t = dp4a_us(nib | (hi << 4), xw[wd], t);
				}
				t -= 32 * xs[k];
				const int sidx = g + 2 * k;
				const int8_t sc = (int8_t)(((sidx < 4 ? Q.sc.x : Q.sc.y) >>
							    (8 * (sidx & 3))) & 0xff);
				tv[k] = __fmul_rn(__fmul_rn(__fmul_rn(dd, (float)sc), xd[k]),
						  __int2float_rn(t));
			}
			*reinterpret_cast<float4 *>(tb + (size_t)r * ts + ((i * 2 + h) * 2 + g) * 4) =
				make_float4(tv[0], tv[1], tv[2], tv[3]);
		}
	};

	pdl_launch_dependents();
	uint32_t G = blockIdx.x;
	if (G < groups)
		load(G, 0);
	pdl_wait();
	{
		// 16-byte chunk c of super-block i: half c / 8, run (k, g) = ((c % 8) / 2,
		// c % 2); its byte sum goes to [i][h][g][k]
		const uint4 *gq = reinterpret_cast<const uint4 *>(p.q);
		for (uint32_t n = threadIdx.x; n < nsb * 16; n += blockDim.x) {
			const uint32_t i = n / 16, c = n % 16, hh = c / 8, kk = (c % 8) / 2, gg = c % 2;
			const uint4 v = gq[n];
			*reinterpret_cast<uint4 *>(aq + (size_t)i * Q6K_ASB + hh * Q6K_AHALF +
						   (c % 8) * 16) = v;
			int sum = dp4a_ss(0x01010101u, v.x, 0);
			sum = dp4a_ss(0x01010101u, v.y, sum);
			sum = dp4a_ss(0x01010101u, v.z, sum);
			sum = dp4a_ss(0x01010101u, v.w, sum);
			xsum[i * 16 + hh * 8 + gg * 4 + kk] = sum;
		}
		for (uint32_t i = threadIdx.x; i < nsb * 8; i += blockDim.x)
			ad[i] = p.d[i];
	}
	__syncthreads();

	for (uint32_t it = 0; G < groups; it++, G += gridDim.x) {
		float *tb = terms + (size_t)(it & 1) * RG * ts;
		for (uint32_t ps = 0; ps < npass; ps++) {
			if (ps)
				load(G, ps);
			compute(ps, tb);
		}
		if (G + gridDim.x < groups)
			load(G + gridDim.x, 0);
		named_barrier(1, W * 32);
		if (warp == 0 && lane < RG) {
			const uint32_t row = G * RG + lane;
			if (row < p.rows) {
				const float4 *t = reinterpret_cast<const float4 *>(tb + (size_t)lane * ts);
				float s = 0.0f;
				for (uint32_t j = 0; j < nsb * 4; j++) {
					const float4 v = t[j];
					s = __fadd_rn(s, v.x);
					s = __fadd_rn(s, v.y);
					s = __fadd_rn(s, v.z);
					s = __fadd_rn(s, v.w);
				}
				p.y[row] = s;
			}
		}
	}
}

} // namespace cgpu
