// SPDX-License-Identifier: GPL-2.0-or-later
// The matvec of charsiu's NPU number format (CHARSIU_NPU_QUANT): int8 weights
// with one fp32 scale a row (npu_tensor_build, reference src/npuquant.c:34-296)
// against an int8 activation with ONE scale d1 (charsiu_act_set's q1,
// src/gguf.c:883-910):
//     acc[r] = sum_k q[r][k] * q1[k]                 (exact int32)
//     y[r]   = (float)acc[r] * d1 * scale[r]         (src/npudev.c:605, 710)
// in float, left to right, as the NPU layer computes it from the accumulator
// the hardware returns. The integer sum is exact in any order, so a warp may
// split a row any way; only the two multiplies are ordered.
//
// Device layout: each tensor's rows back to back, a row padded with zeros to
// kp bytes (kp = K rounded up to 16), so a lane's 16-byte loads are aligned.
// The grid's warps split the rows into contiguous ranges of equal size (to a
// row), so every SM carries the same bytes; a warp takes its range up to R
// rows at a time (rows_per_warp, chosen by the host); lane L reads 16-byte chunks
// L, L + 32, ... of each, U chunks of each row per step (R * U <= 16 loads in
// flight a lane), and dots them with dp4a against the activation staged in
// shared memory; one warp reduction a row, and lane j writes row j. The first
// rows' first chunks are loaded before the wait on the previous kernel, and
// each next batch's while the current one's sums are reduced.
#pragma once

#include <cstdint>

#include "ptx.cuh"

namespace cgpu {

constexpr int NPU_MAX_TENSORS = 8;
constexpr int NPU_WARPS = 8;
constexpr int NPU_INLINE_WORDS = 896;        // the activation in kernel parameters, up to K = 14336

struct NpuTensor {
	const int8_t *w;         // [rows][kp]
	const float *scale;      // [rows]
	float *y;
	uint32_t rows, row_end;  // row_end: rows of this and every tensor before it
};

struct NpuParams {
	NpuTensor t[NPU_MAX_TENSORS];
	uint32_t ntensor, total_rows, kp;
	uint32_t rows_per_warp;  // 1 .. the kernel's R
	float d1;
	const float *d1p;        // when set, d1 is read here (device) once the kernel before is done
	const int8_t *q1;        // kp bytes (device); unused when the activation is inline
	// direct host calls: when done_flag is set, the last CTA to finish
	// writes `seq` there (mapped host memory) once every y is visible to the
	// host, and the kernel time since *t_start + 1
	uint32_t *done_count;
	uint32_t *done_flag;
	unsigned long long *t_start;
	uint32_t seq;
};

// The activation carried in the launch's parameters (a direct host call):
// kp bytes in 16-byte words.
template <int AW>
struct NpuInline {
	NpuParams p;
	uint4 act[AW];
};
static_assert(sizeof(NpuInline<NPU_INLINE_WORDS>) <= 32764, "kernel parameter space");

__device__ __forceinline__ int dp4a_s(uint32_t a, uint32_t b, int c)
{
	return __dp4a((int)a, (int)b, c);
}

template <int R, int U, int AW>
__device__ __forceinline__ void npumv_body(const NpuParams &p, const uint4 *inl)
{
	extern __shared__ __align__(16) uint8_t npu_smem[];
	const uint32_t nch = p.kp / 16;
	uint4 *act = reinterpret_cast<uint4 *>(npu_smem);
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const uint32_t nw = gridDim.x * NPU_WARPS;

	// rows r0 .. r0 + R - 1 of this warp's range [r0, r_end): their tensors
	// and row pointers
	const uint32_t rpw = p.rows_per_warp;
	const uint32_t gw = blockIdx.x * NPU_WARPS + warp;
	const uint32_t r_end = (uint32_t)((uint64_t)(gw + 1) * p.total_rows / nw);
	const int8_t *wr[R];
	uint32_t ti[R];
	auto setup = [&](uint32_t r0) {
#pragma unroll
		for (int j = 0; j < R; j++) {
			const uint32_t r = r0 + j;
			uint32_t t = 0;
			while (t + 1 < p.ntensor && r >= p.t[t].row_end)
				t++;
			ti[j] = t;
			wr[j] = ((uint32_t)j < rpw && r < r_end)
				? p.t[t].w + (uint64_t)(r - (p.t[t].row_end - p.t[t].rows)) * p.kp
				: nullptr;
		}
	};
	uint4 wv[R][U];
	auto load = [&](uint32_t c0) {
#pragma unroll
		for (int j = 0; j < R; j++)
#pragma unroll
			for (int u = 0; u < U; u++) {
				const uint32_t c = c0 + 32 * u;
				wv[j][u] = (wr[j] && c < nch) ? ldg_stream((const uint8_t *)wr[j] + c * 16)
							     : make_uint4(0, 0, 0, 0);
			}
	};

	// the first rows' first chunks go now: weights never depend on the
	// kernel before this one
	if (rpw < 1 || rpw > (uint32_t)R)
		return;
	uint32_t r0 = (uint32_t)((uint64_t)gw * p.total_rows / nw);
	setup(r0);
	load(lane);
	if (AW && p.done_flag && blockIdx.x == 0 && threadIdx.x == 0)
		*p.t_start = globaltimer_ns();
	if (AW) {
		for (uint32_t i = threadIdx.x; i < nch; i += blockDim.x)
			act[i] = inl[i];
	}
	pdl_wait();
	if (!AW) {
		const uint4 *g4 = reinterpret_cast<const uint4 *>(p.q1);
		for (uint32_t i = threadIdx.x; i < nch; i += blockDim.x)
			act[i] = g4[i];
	}
	const float d1 = p.d1p ? *p.d1p : p.d1;
	__syncthreads();
	pdl_launch_dependents();

	while (r0 < r_end) {
		int acc[R];
#pragma unroll
		for (int j = 0; j < R; j++)
			acc[j] = 0;
		for (uint32_t c0 = lane; c0 < nch; c0 += 32 * U) {
			if (c0 != (uint32_t)lane)
				load(c0);
#pragma unroll
			for (int u = 0; u < U; u++) {
				const uint32_t c = c0 + 32 * u;
				if (c < nch) {
					const uint4 a = act[c];
#pragma unroll
					for (int j = 0; j < R; j++) {
						acc[j] = dp4a_s(wv[j][u].x, a.x, acc[j]);
						acc[j] = dp4a_s(wv[j][u].y, a.y, acc[j]);
						acc[j] = dp4a_s(wv[j][u].z, a.z, acc[j]);
						acc[j] = dp4a_s(wv[j][u].w, a.w, acc[j]);
					}
				}
			}
		}
		// where this batch's rows go, then the next batch's first chunks in
		// flight while this one's sums are reduced and stored
		float *yp[R];
		float sc[R];
#pragma unroll
		for (int j = 0; j < R; j++) {
			yp[j] = nullptr;
			sc[j] = 0.0f;
			if (lane == j && wr[j]) {
				const NpuTensor &t = p.t[ti[j]];
				const uint32_t row = r0 + j - (t.row_end - t.rows);
				yp[j] = t.y + row;
				sc[j] = t.scale[row];
			}
		}
		r0 += rpw;
		setup(r0);
		load(lane);
#pragma unroll
		for (int j = 0; j < R; j++) {
			const int s = __reduce_add_sync(0xffffffffu, acc[j]);
			if (yp[j])
				*yp[j] = __fmul_rn(__fmul_rn(__int2float_rn(s), d1), sc[j]);
		}
	}
	if (AW && p.done_flag) {
		// y is mapped host memory: this CTA's stores reach thread 0 through
		// the barrier and are released at device scope by its count; the
		// last CTA acquires them all and orders them before the flag with one
		// system fence
		__syncthreads();
		if (threadIdx.x == 0 && atom_add_acq_rel_gpu(p.done_count, 1u) == gridDim.x - 1) {
			*p.done_count = 0;
			const unsigned long long dt =
				globaltimer_ns() - *(volatile const unsigned long long *)p.t_start;
			__threadfence_system();
			p.done_flag[1] = dt > 0xffffffffull ? 0xffffffffu : (uint32_t)dt;
			__threadfence_system();
			*(volatile uint32_t *)p.done_flag = p.seq;
		}
	}
}

template <int R, int U>
__global__ void __launch_bounds__(NPU_WARPS * 32)
npumv_kernel(const __grid_constant__ NpuParams p)
{
	npumv_body<R, U, 0>(p, nullptr);
}

template <int R, int U, int AW>
__global__ void __launch_bounds__(NPU_WARPS * 32)
npumv_inline_kernel(const __grid_constant__ NpuInline<AW> a)
{
	npumv_body<R, U, AW>(a.p, a.act);
}

} // namespace cgpu
