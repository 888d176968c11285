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
// 16 bytes. Lane L of a warp takes super-block i0 + L/4, half (L/2)&1 and
// g = L&1 -- three 16-byte loads, one 8-byte load of the half's scales -- and
// computes its four terms with dp4a (unsigned 6-bit weights, so the -32 comes
// off as 32 * sum(activation)). A warp takes up to 8 rows at a time (fewer
// when the tensor has too few rows to fill the GPU): the terms of each row's
// 8 super-blocks go to that row's line of a per-warp buffer, then lane r adds
// row r's line in term order -- the reference's sequence -- so the ordered
// sums run side by side (a lane-0 sum of one row at a time is 12% slower on
// the head). Each item's bytes are loaded two items ahead.
#pragma once

#include "layout.h"
#include "ptx.cuh"
#include "qmv1.cuh"

namespace cgpu {

constexpr int Q6K_WARPS = 8;
// rows a warp sums side by side (lane r: row r). Measured on the 2048 x 128256
// head: 1 (a lane-0 sum) 74 us, 4 70 us, 8 66 us, 16 92 us (its term buffers
// cost occupancy).
constexpr int Q6K_ROWS = 8;
constexpr int Q6K_TSTRIDE = 129;      // floats a row of the term buffer: 128 + 1 (banks)

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
	uint32_t rows_per_warp;    // 1 .. Q6K_ROWS: rows a warp sums side by side
	const int8_t *q;           // activation [nsb * 256]
	const float *d;            // activation deltas [nsb * 8]
};

inline size_t q6k_smem_bytes(uint32_t nsb)
{
	return (size_t)nsb * 256 + (size_t)nsb * 8 * sizeof(float) +
	       (size_t)Q6K_WARPS * Q6K_ROWS * Q6K_TSTRIDE * sizeof(float);
}

__global__ void __launch_bounds__(Q6K_WARPS * 32)
q6k_kernel(const __grid_constant__ Q6kParams p)
{
	extern __shared__ __align__(128) uint8_t smem[];
	const uint32_t nsb = p.nsb;
	int8_t *aq = reinterpret_cast<int8_t *>(smem);
	float *ad = reinterpret_cast<float *>(smem + (size_t)nsb * 256);
	float *terms = ad + (size_t)nsb * 8;

	pdl_wait();
	{
		const uint4 *gq = reinterpret_cast<const uint4 *>(p.q);
		uint4 *sq = reinterpret_cast<uint4 *>(aq);
		for (uint32_t i = threadIdx.x; i < nsb * 16; i += blockDim.x)
			sq[i] = gq[i];
		for (uint32_t i = threadIdx.x; i < nsb * 8; i += blockDim.x)
			ad[i] = p.d[i];
	}
	__syncthreads();
	pdl_launch_dependents();

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const uint32_t h = (lane >> 1) & 1, g = lane & 1;
	const uint64_t rs = q6k_row_bytes(nsb);
	float *tw = terms + warp * Q6K_ROWS * Q6K_TSTRIDE;
	if (p.rows_per_warp < 1 || p.rows_per_warp > (uint32_t)Q6K_ROWS)
		return;

	// one item = (row, 8 super-blocks from i0); items go in the order (rows
	// base.. base + nr - 1 of a chunk, chunk, base), and each item's bytes are
	// loaded two items ahead
	struct Regs {
		uint4 ql0, ql1, qh;
		uint2 sc;
		uint16_t d;
	};
	struct Cursor {
		uint32_t base, i0, r;
	};
	const uint32_t rpw = p.rows_per_warp;
	const uint32_t step = gridDim.x * Q6K_WARPS * rpw;
	auto rows_at = [&](uint32_t base) { return p.rows - base < rpw ? p.rows - base : rpw; };
	auto advance = [&](Cursor &c) {
		if (++c.r == rows_at(c.base)) {
			c.r = 0;
			c.i0 += 8;
			if (c.i0 >= nsb) {
				c.i0 = 0;
				c.base += step;
			}
		}
	};
	auto load = [&](const Cursor &c, Regs &R) {
		const uint32_t i = c.i0 + (lane >> 2);
		if (i >= nsb)
			return;
		const uint8_t *wr = p.w + (uint64_t)(c.base + c.r) * rs;
		const uint8_t *sb = wr + (size_t)i * 208;
		R.ql0 = ldg_stream(sb + h * 64 + g * 16);
		R.ql1 = ldg_stream(sb + h * 64 + 32 + g * 16);
		R.qh = ldg_stream(sb + 128 + h * 32 + g * 16);
		R.sc = *reinterpret_cast<const uint2 *>(sb + 192 + h * 8);
		R.d = ldg_stream_u16(wr + (size_t)nsb * 208 + 2 * i);
	};
	Cursor cc = {(blockIdx.x * Q6K_WARPS + warp) * rpw, 0, 0};
	Cursor lc = cc;
	Regs r0 = {}, r1 = {}, r2 = {};
	if (lc.base < p.rows) {
		load(lc, r0);
		advance(lc);
	}
	if (lc.base < p.rows) {
		load(lc, r1);
		advance(lc);
	}
	float s = 0.0f;
	while (cc.base < p.rows) {
		if (lc.base < p.rows) {
			load(lc, r2);
			advance(lc);
		}
		const uint32_t i = cc.i0 + (lane >> 2);
		float tv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
		if (i < nsb) {
			const float dd = half_bits_to_float(r0.d);
			const int8_t *xq = aq + (size_t)i * 256 + h * 128 + g * 16;
			const float *xd = ad + (size_t)i * 8 + h * 4;
			const uint32_t ql0w[4] = {r0.ql0.x, r0.ql0.y, r0.ql0.z, r0.ql0.w};
			const uint32_t ql1w[4] = {r0.ql1.x, r0.ql1.y, r0.ql1.z, r0.ql1.w};
			const uint32_t qhw[4] = {r0.qh.x, r0.qh.y, r0.qh.z, r0.qh.w};
#pragma unroll
			for (int k = 0; k < 4; k++) {
				int t = 0, xs = 0;
				const uint32_t *x4 = reinterpret_cast<const uint32_t *>(xq + k * 32);
#pragma unroll
				for (int wd = 0; wd < 4; wd++) {
					const uint32_t lo = (k & 1) ? ql1w[wd] : ql0w[wd];
					const uint32_t nib = (k & 2) ? (lo >> 4) & 0x0f0f0f0fu
								     : lo & 0x0f0f0f0fu;
					const uint32_t hi = (qhw[wd] >> (2 * k)) & 0x03030303u;
					const uint32_t x = x4[wd];
					t = dp4a_us(nib | (hi << 4), x, t);
					xs = dp4a_ss(0x01010101u, x, xs);
				}
				t -= 32 * xs;
				const int sidx = g + 2 * k;
				const int8_t sc = (int8_t)(((sidx < 4 ? r0.sc.x : r0.sc.y) >>
							    (8 * (sidx & 3))) & 0xff);
				tv[k] = __fmul_rn(__fmul_rn(__fmul_rn(dd, (float)sc), xd[k]),
						  __int2float_rn(t));
			}
		}
		// term lane * 4 + k of the chunk at [r][k * 32 + lane]
#pragma unroll
		for (int k = 0; k < 4; k++)
			tw[cc.r * Q6K_TSTRIDE + k * 32 + lane] = tv[k];
		const uint32_t nr = rows_at(cc.base);
		if (cc.r + 1 == nr) {
			// the chunk of every row of this base is in: lane r adds row r's
			__syncwarp();
			if ((uint32_t)lane < nr) {
				const uint32_t nl = (nsb - cc.i0 < 8 ? nsb - cc.i0 : 8) * 4;
				const float *t = tw + lane * Q6K_TSTRIDE;
				for (uint32_t l = 0; l < nl; l++)
#pragma unroll
					for (int k = 0; k < 4; k++)
						s = __fadd_rn(s, t[k * 32 + l]);
				if (cc.i0 + 8 >= nsb) {
					p.y[cc.base + lane] = s;
					s = 0.0f;
				}
			}
			__syncwarp();
		}
		r0 = r1;
		r1 = r2;
		advance(cc);
	}
}

} // namespace cgpu
