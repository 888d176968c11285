// SPDX-License-Identifier: GPL-2.0-or-later
// The block-quant matvec: y = W x for q8_0 / q4_0 W and a q8_0 activation,
// bit-identical to charsiu's gguf_matvec (reference src/gguf.c:1061-1107,
// 1149-1171).
//
// The reference's arithmetic per output row is
//     s = 0; for b in blocks: s += (d_w[b] * d_a[b]) * (float)t_b
// with t_b the exact int32 dot of block b, every multiply and add rounded on
// its own, left to right. Integer dots can be split any way; the float sum
// cannot. So each 8-row group is owned by ONE warp that walks the group's K
// in block order, and each row's running sum lives in one lane. Parallelism
// comes from many groups (RG = 8 rows keeps even N = 512 at 64 groups).
//
// Data movement: each warp owns a ring of QMV_STAGES shared-memory stages; its
// lane 0 issues one single-destination bulk copy (cp.async.bulk) per segment of 16
// blocks x 8 rows (4352 bytes q8_0, 2304 q4_0) and the warp consumes stages in
// order, refilling each as soon as it is read. The weights do not depend on
// the previous kernel, so the ring is filled before griddepcontrol.wait; only
// the activation waits for it.
#pragma once

#include "layout.h"
#include "ptx.cuh"

namespace cgpu {

constexpr int QMV_WARPS = 4;
constexpr int QMV_STAGES = 5;
constexpr int QMV_MAX_TENSORS = 8;
constexpr int QMV_MAX_M = 8;

struct QmvTensor {
	const uint8_t *data;     // the device layout of layout.h
	float *y;                // y[m * y_stride + row], rows of this GPU
	uint32_t type, rows, groups, group_end;
	uint32_t y_stride;
	uint32_t pad_;
};

struct QmvParams {
	QmvTensor t[QMV_MAX_TENSORS];
	uint32_t ntensor, total_groups, k, nb;
	const int8_t *q;         // activation quants [M][nb * 32]
	const float *d;          // activation deltas [M][nb]
	int *err;                // set nonzero if a wait gave up (mapped host memory)
	// direct host calls (M = 1): when done_flag is set, the last CTA to
	// finish writes `seq` there (mapped host memory) once every y is visible
	// to the host, and the kernel time since *t_start there + 1
	uint32_t *done_count;    // device, zero between launches
	uint32_t *done_flag;     // [0] seq, [1] kernel ns
	unsigned long long *t_start;
	uint32_t seq;
};

inline size_t qmv_smem_bytes(int m, uint32_t nb)
{
	return (size_t)QMV_WARPS * QMV_STAGES * MAX_SEG_BYTES +
	       (size_t)QMV_WARPS * QMV_STAGES * sizeof(uint64_t) +
	       (size_t)m * nb * (32 + sizeof(float) + sizeof(int32_t));
}

// One segment (sb <= 16 blocks of 8 rows), in two phases. Lane l owns block
// p = l>>3 of every 4-block step and row r = l&7; it computes the terms
// (d_w * d_a) * t of its blocks with no dependence between them, so the
// loads, dp4a and multiplies of all steps overlap. Then lane r adds row r's
// terms in block order (step by step, blocks p = 0..3 fetched by shuffle),
// which is the only serial part: one fadd per block.
//
// q8_0: a block row is two 16-byte chunks (layout.h), 8 lanes of one chunk
// reading 128 contiguous bytes. q4_0: a block row is 16 bytes of nibbles;
// (q - 8) . a = q . a - 8 * sum(a).
template <int M, bool Q8>
__device__ __forceinline__ void seg_terms(const uint8_t *st, uint32_t sb, uint32_t b0,
					  const int8_t *aq, const float *ad, const int32_t *asum,
					  uint32_t nb, int lane, float (&s)[M])
{
	constexpr uint32_t QB = Q8 ? 32 : 16;
	const uint16_t *dl = reinterpret_cast<const uint16_t *>(st + sb * RG * QB);
	const int p = lane >> 3, r = lane & 7;
	float term[SB / 4][M];

#pragma unroll
	for (int j = 0; j < SB / 4; j++) {
		if ((uint32_t)j * 4 >= sb)
			break;
		const uint32_t bl = min((uint32_t)(j * 4 + p), sb - 1);
		const uint32_t blk = b0 + bl;
		const uint8_t *wp = st + bl * RG * QB + r * 16;
		const float dw = half_bits_to_float(dl[bl * RG + r]);
		if (Q8) {
			const uint4 w0 = *reinterpret_cast<const uint4 *>(wp);
			const uint4 w1 = *reinterpret_cast<const uint4 *>(wp + RG * 16);
#pragma unroll
			for (int m = 0; m < M; m++) {
				const int8_t *a = aq + ((size_t)m * nb + blk) * 32;
				const uint4 a0 = *reinterpret_cast<const uint4 *>(a);
				const uint4 a1 = *reinterpret_cast<const uint4 *>(a + 16);
				int t0 = dp4a_ss(w0.x, a0.x, 0), t1 = dp4a_ss(w1.x, a1.x, 0);
				t0 = dp4a_ss(w0.y, a0.y, t0);
				t1 = dp4a_ss(w1.y, a1.y, t1);
				t0 = dp4a_ss(w0.z, a0.z, t0);
				t1 = dp4a_ss(w1.z, a1.z, t1);
				t0 = dp4a_ss(w0.w, a0.w, t0);
				t1 = dp4a_ss(w1.w, a1.w, t1);
				term[j][m] = __fmul_rn(__fmul_rn(dw, ad[m * nb + blk]),
						       __int2float_rn(t0 + t1));
			}
		} else {
			const uint4 w = *reinterpret_cast<const uint4 *>(wp);
			const uint32_t l0 = w.x & 0x0f0f0f0fu, l1 = w.y & 0x0f0f0f0fu;
			const uint32_t l2 = w.z & 0x0f0f0f0fu, l3 = w.w & 0x0f0f0f0fu;
			const uint32_t h0 = (w.x >> 4) & 0x0f0f0f0fu, h1 = (w.y >> 4) & 0x0f0f0f0fu;
			const uint32_t h2 = (w.z >> 4) & 0x0f0f0f0fu, h3 = (w.w >> 4) & 0x0f0f0f0fu;
#pragma unroll
			for (int m = 0; m < M; m++) {
				const uint4 *ap = reinterpret_cast<const uint4 *>(aq + ((size_t)m * nb + blk) * 32);
				const uint4 a0 = ap[0], a1 = ap[1];
				int t0 = dp4a_us(l0, a0.x, 0), t1 = dp4a_us(h0, a1.x, 0);
				t0 = dp4a_us(l1, a0.y, t0);
				t1 = dp4a_us(h1, a1.y, t1);
				t0 = dp4a_us(l2, a0.z, t0);
				t1 = dp4a_us(h2, a1.z, t1);
				t0 = dp4a_us(l3, a0.w, t0);
				t1 = dp4a_us(h3, a1.w, t1);
				term[j][m] = __fmul_rn(__fmul_rn(dw, ad[m * nb + blk]),
						       __int2float_rn(t0 + t1 - 8 * asum[m * nb + blk]));
			}
		}
	}
#pragma unroll
	for (int j = 0; j < SB / 4; j++) {
		if ((uint32_t)j * 4 >= sb)
			break;
#pragma unroll
		for (int m = 0; m < M; m++) {
			const float t1 = __shfl_sync(0xffffffffu, term[j][m], r + 8);
			const float t2 = __shfl_sync(0xffffffffu, term[j][m], r + 16);
			const float t3 = __shfl_sync(0xffffffffu, term[j][m], r + 24);
			s[m] = __fadd_rn(s[m], term[j][m]);
			if ((uint32_t)j * 4 + 1 < sb)
				s[m] = __fadd_rn(s[m], t1);
			if ((uint32_t)j * 4 + 2 < sb)
				s[m] = __fadd_rn(s[m], t2);
			if ((uint32_t)j * 4 + 3 < sb)
				s[m] = __fadd_rn(s[m], t3);
		}
	}
}

template <int M>
__global__ void __launch_bounds__(QMV_WARPS * 32)
qmv_kernel(const __grid_constant__ QmvParams p)
{
	extern __shared__ __align__(128) uint8_t smem[];
	uint64_t *bars = reinterpret_cast<uint64_t *>(smem + QMV_WARPS * QMV_STAGES * MAX_SEG_BYTES);
	int8_t *aq = reinterpret_cast<int8_t *>(bars + QMV_WARPS * QMV_STAGES);
	const uint32_t nb = p.nb;
	float *ad = reinterpret_cast<float *>(aq + (size_t)M * nb * 32);
	int32_t *asum = reinterpret_cast<int32_t *>(ad + (size_t)M * nb);

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	uint8_t *ring = smem + (size_t)warp * QMV_STAGES * MAX_SEG_BYTES;
	uint64_t *bar = bars + warp * QMV_STAGES;

	// groups are dealt to warps round robin across CTAs first, so a small
	// projection still spreads over every SM
	const uint32_t gw = warp * gridDim.x + blockIdx.x;
	const uint32_t tw = QMV_WARPS * gridDim.x;
	const uint32_t nseg = nsegments(nb);
	const uint32_t my_groups = gw < p.total_groups ? (p.total_groups - gw + tw - 1) / tw : 0;
	const uint32_t nitems = my_groups * nseg;

	auto locate = [&](uint32_t item, uint32_t &ti, uint32_t &lg, uint32_t &seg) {
		const uint32_t G = gw + (item / nseg) * tw;
		seg = item % nseg;
		ti = 0;
		while (ti + 1 < p.ntensor && G >= p.t[ti].group_end)
			ti++;
		lg = G - (p.t[ti].group_end - p.t[ti].groups);
	};
	auto issue = [&](uint32_t item) {
		uint32_t ti, lg, seg;
		locate(item, ti, lg, seg);
		const QmvTensor &T = p.t[ti];
		const uint32_t bytes = seg_blocks(nb, seg) * block_group_bytes(T.type);
		const uint8_t *src = T.data + (uint64_t)lg * group_bytes(T.type, nb) +
				     seg_offset(T.type, seg);
		uint64_t *b = &bar[item % QMV_STAGES];
		mbar_arrive_expect_tx(b, bytes);
		bulk_g2s(ring + (item % QMV_STAGES) * MAX_SEG_BYTES, src, bytes, b);
	};

	if (lane == 0) {
		for (int i = 0; i < QMV_STAGES; i++)
			mbar_init(&bar[i], 1);
		fence_mbar_init();
		const uint32_t pre = nitems < QMV_STAGES ? nitems : QMV_STAGES;
		for (uint32_t i = 0; i < pre; i++)
			issue(i);
	}

	// the activation is the previous kernel's output; wait for it only now
	pdl_wait();
	{
		const uint32_t n16 = M * nb * 2;
		const uint4 *gq = reinterpret_cast<const uint4 *>(p.q);
		uint4 *sq = reinterpret_cast<uint4 *>(aq);
		for (uint32_t i = threadIdx.x; i < n16; i += blockDim.x)
			sq[i] = gq[i];
		for (uint32_t i = threadIdx.x; i < M * nb; i += blockDim.x)
			ad[i] = p.d[i];
	}
	__syncthreads();
	for (uint32_t i = threadIdx.x; i < M * nb; i += blockDim.x) {
		const uint4 *b = reinterpret_cast<const uint4 *>(aq + (size_t)i * 32);
		const uint4 u = b[0], v = b[1];
		int sum = dp4a_ss(u.x, 0x01010101u, 0);
		sum = dp4a_ss(u.y, 0x01010101u, sum);
		sum = dp4a_ss(u.z, 0x01010101u, sum);
		sum = dp4a_ss(u.w, 0x01010101u, sum);
		sum = dp4a_ss(v.x, 0x01010101u, sum);
		sum = dp4a_ss(v.y, 0x01010101u, sum);
		sum = dp4a_ss(v.z, 0x01010101u, sum);
		sum = dp4a_ss(v.w, 0x01010101u, sum);
		asum[i] = sum;
	}
	__syncthreads();
	pdl_launch_dependents();

	float s[M];
#pragma unroll
	for (int m = 0; m < M; m++)
		s[m] = 0.0f;

	for (uint32_t i = 0; i < nitems; i++) {
		const uint32_t stage = i % QMV_STAGES;
		if (!mbar_wait_bounded(&bar[stage], (i / QMV_STAGES) & 1, WAIT_LIMIT_NS)) {
			if (lane == 0)
				*(volatile int *)p.err = 1;
			// let the copies already issued land before this CTA leaves
			const uint32_t issued = min(nitems, i + QMV_STAGES);
			for (uint32_t j = i + 1; j < issued; j++)
				mbar_wait_bounded(&bar[j % QMV_STAGES], (j / QMV_STAGES) & 1, WAIT_LIMIT_NS);
			return;
		}
		uint32_t ti, lg, seg;
		locate(i, ti, lg, seg);
		const QmvTensor &T = p.t[ti];
		if (seg == 0) {
#pragma unroll
			for (int m = 0; m < M; m++)
				s[m] = 0.0f;
		}
		const uint8_t *st = ring + stage * MAX_SEG_BYTES;
		const uint32_t sb = seg_blocks(nb, seg);
		if (T.type == TYPE_Q8_0)
			seg_terms<M, true>(st, sb, seg * SB, aq, ad, asum, nb, lane, s);
		else
			seg_terms<M, false>(st, sb, seg * SB, aq, ad, asum, nb, lane, s);
		__syncwarp();
		if (lane == 0 && i + QMV_STAGES < nitems) {
			fence_proxy_async_smem();
			issue(i + QMV_STAGES);
		}
		if (seg == nseg - 1) {
			const uint32_t row = lg * RG + lane;
			if (lane < RG && row < T.rows) {
#pragma unroll
				for (int m = 0; m < M; m++)
					T.y[(size_t)m * T.y_stride + row] = s[m];
			}
		}
	}
}

} // namespace cgpu
