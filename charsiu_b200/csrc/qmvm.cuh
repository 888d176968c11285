// SPDX-License-Identifier: GPL-2.0-or-later
// The block-quant matvec of a few activations (M = 2, 4, 8) on the CUDA
// cores: qmv1.cuh's organisation, each lane's weights used M times.
//
// Same arithmetic as qmv.cuh (bit-identical to charsiu's gguf_matvec of each
// activation, reference src/gguf.c:1061-1107, 1149-1171). A CTA of W warps
// owns one 8-row group at a time over a persistent grid; the group's 16-block
// segments are split over the warps (one or, with TWO, two a warp) and loaded
// straight into registers with 16-byte non-allocating loads, the first
// group's before griddepcontrol.wait. Lane l owns block l>>3 of every 4-block
// step and row l&7: from its weight registers it computes the exact int32 dot
// with each of the M activations (dp4a) and the term (d_w * d_a) * t, into a
// per-activation term buffer in shared memory. One named barrier per group;
// then M * 8 threads -- one per (activation, row) -- add their terms in block
// order and store y, while the other warps already load the next group into
// the other term buffer.
//
// The term buffer of one activation is padded by 8 floats so that the 32
// summing lanes of a warp (4 activations x 8 rows) hit 32 different banks.
#pragma once

#include "layout.h"
#include "ptx.cuh"
#include "qmv.cuh"
#include "qmv1.cuh"

namespace cgpu {

__host__ __device__ constexpr uint32_t qmvm_term_stride(uint32_t nb)
{
	return nb * RG + 8;
}

inline size_t qmvm_smem_bytes(int m, uint32_t nb)
{
	return (size_t)2 * m * qmvm_term_stride(nb) * sizeof(float) +
	       (size_t)m * nb * (32 + sizeof(float) + sizeof(int32_t));
}

// One segment of one group for M activations: lane (p = l>>3, r = l&7) and
// 4-block step j hold block bl = 4j + p of row r in registers (seg_load).
template <bool Q8, int M>
__device__ __forceinline__ void segm_compute(const SegRegs<Q8> &R, uint32_t sb, uint32_t b0,
					     const int8_t *aq, const float *ad, const int32_t *asum,
					     uint32_t nb, int lane, float *tb)
{
	const int p = lane >> 3, r = lane & 7;
	const uint32_t ts = qmvm_term_stride(nb);
#pragma unroll
	for (int j = 0; j < SB / 4; j++) {
		const uint32_t bl = (uint32_t)(j * 4 + p);
		if ((uint32_t)j * 4 >= sb)
			break;
		if (bl >= sb)
			continue;
		const uint32_t blk = b0 + bl;
		const float dw = half_bits_to_float(R.dl[j]);
#pragma unroll
		for (int a = 0; a < M; a++) {
			const uint4 *ap = reinterpret_cast<const uint4 *>(aq + ((size_t)a * nb + blk) * 32);
			const uint4 a0 = ap[0], a1 = ap[1];
			int t;
			if (Q8) {
				const uint4 w0 = R.w[j][0], w1 = R.w[j][Q8 ? 1 : 0];
				int t0 = dp4a_ss(w0.x, a0.x, 0), t1 = dp4a_ss(w1.x, a1.x, 0);
				t0 = dp4a_ss(w0.y, a0.y, t0);
				t1 = dp4a_ss(w1.y, a1.y, t1);
				t0 = dp4a_ss(w0.z, a0.z, t0);
				t1 = dp4a_ss(w1.z, a1.z, t1);
				t0 = dp4a_ss(w0.w, a0.w, t0);
				t1 = dp4a_ss(w1.w, a1.w, t1);
				t = t0 + t1;
			} else {
				const uint4 w = R.w[j][0];
				int t0 = dp4a_us(w.x & 0x0f0f0f0fu, a0.x, 0);
				int t1 = dp4a_us((w.x >> 4) & 0x0f0f0f0fu, a1.x, 0);
				t0 = dp4a_us(w.y & 0x0f0f0f0fu, a0.y, t0);
				t1 = dp4a_us((w.y >> 4) & 0x0f0f0f0fu, a1.y, t1);
				t0 = dp4a_us(w.z & 0x0f0f0f0fu, a0.z, t0);
				t1 = dp4a_us((w.z >> 4) & 0x0f0f0f0fu, a1.z, t1);
				t0 = dp4a_us(w.w & 0x0f0f0f0fu, a0.w, t0);
				t1 = dp4a_us((w.w >> 4) & 0x0f0f0f0fu, a1.w, t1);
				t = t0 + t1 - 8 * asum[a * nb + blk];
			}
			tb[a * ts + blk * RG + r] =
				__fmul_rn(__fmul_rn(dw, ad[a * nb + blk]), __int2float_rn(t));
		}
	}
}

// W warps a CTA, one quant type a launch (Q8), segments as qmv1_kernel.
template <int W, bool Q8, bool TWO, int M>
__global__ void __launch_bounds__(W * 32)
qmvm_kernel(const __grid_constant__ QmvParams p)
{
	static_assert(M * RG <= W * 32, "one summing thread per (activation, row)");
	extern __shared__ __align__(128) uint8_t smem[];
	const uint32_t nb = p.nb, ts = qmvm_term_stride(nb);
	float *terms = reinterpret_cast<float *>(smem);
	int8_t *aq = reinterpret_cast<int8_t *>(terms + (size_t)2 * M * ts);
	float *ad = reinterpret_cast<float *>(aq + (size_t)M * nb * 32);
	int32_t *asum = reinterpret_cast<int32_t *>(ad + (size_t)M * nb);
	constexpr uint32_t QB = Q8 ? 32 : 16;

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const uint32_t nseg = nsegments(nb);
	const uint32_t s0 = warp, s1 = warp + W;

	auto locate = [&](uint32_t G, uint32_t &ti, uint32_t &lg) {
		ti = 0;
		while (ti + 1 < p.ntensor && G >= p.t[ti].group_end)
			ti++;
		lg = G - (p.t[ti].group_end - p.t[ti].groups);
	};
	auto seg_ptr = [&](uint32_t ti, uint32_t lg, uint32_t seg) {
		return p.t[ti].data + (uint64_t)lg * nb * (RG * (QB + 2)) +
		       (uint64_t)seg * SB * (RG * (QB + 2));
	};
	SegRegs<Q8> R0, R1;
	auto load = [&](uint32_t G) {
		uint32_t ti, lg;
		locate(G, ti, lg);
		if (s0 < nseg)
			seg_load<Q8>(R0, seg_ptr(ti, lg, s0), seg_blocks(nb, s0), lane);
		if (TWO && s1 < nseg)
			seg_load<Q8>(R1, seg_ptr(ti, lg, s1), seg_blocks(nb, s1), lane);
	};

	// weights do not depend on the previous kernel: the first group's go now
	uint32_t G = blockIdx.x;
	if (G < p.total_groups)
		load(G);

	pdl_wait();
	{
		// the M activations are consecutive rows [M][nb * 32] and [M][nb]
		const uint4 *gq = reinterpret_cast<const uint4 *>(p.q);
		uint4 *sq = reinterpret_cast<uint4 *>(aq);
		for (uint32_t i = threadIdx.x; i < (uint32_t)M * nb * 2; i += blockDim.x)
			sq[i] = gq[i];
		for (uint32_t i = threadIdx.x; i < (uint32_t)M * nb; i += blockDim.x)
			ad[i] = p.d[i];
	}
	__syncthreads();
	if (!Q8) {
		for (uint32_t i = threadIdx.x; i < (uint32_t)M * nb; i += blockDim.x) {
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
	}
	pdl_launch_dependents();

	for (uint32_t i = 0; G < p.total_groups; i++, G += gridDim.x) {
		uint32_t ti, lg;
		locate(G, ti, lg);
		float *tb = terms + (size_t)(i & 1) * M * ts;
		if (s0 < nseg)
			segm_compute<Q8, M>(R0, seg_blocks(nb, s0), s0 * SB, aq, ad, asum, nb, lane, tb);
		if (TWO && s1 < nseg)
			segm_compute<Q8, M>(R1, seg_blocks(nb, s1), s1 * SB, aq, ad, asum, nb, lane, tb);
		// the registers are free: the next group's weights go now, in flight
		// through the barrier and the in-order sums below
		if (G + gridDim.x < p.total_groups)
			load(G + gridDim.x);
		named_barrier(1, W * 32);
		if (threadIdx.x < (unsigned)(M * RG)) {
			const uint32_t a = threadIdx.x / RG, r = threadIdx.x % RG;
			const float *t = tb + a * ts + r;
			float s = 0.0f;
#pragma unroll 16
			for (uint32_t b = 0; b < nb; b++)
				s = __fadd_rn(s, t[b * RG]);
			const uint32_t row = lg * RG + r;
			const QmvTensor &T = p.t[ti];
			if (row < T.rows)
				T.y[(uint64_t)a * T.y_stride + row] = s;
		}
	}
}

} // namespace cgpu
