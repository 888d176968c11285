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
//
// Organised as the q8_0 decode matvec (qmv1.cuh): rows in 8-row groups dealt
// round robin over a persistent grid of small CTAs (up to eight an SM at
// K = 2048), the W warps of a CTA splitting K. Chunk c (16 bytes) of a row is
// read by warp (c / 32) % W, lane c % 32, in register slot (c / 32W) % U of
// pass c / (32WU), so every warp-load instruction reads 512 contiguous bytes
// of one row and a lane holds one chunk of each of the group's 8 rows a slot.
// A row's warp partial is one __reduce_add_sync; the W partials meet in
// shared memory (int32: exact in any order) and thread j of the CTA scales
// row j. The first group's loads go out before the wait on the previous
// kernel, each next group's as soon as the current group's are consumed, so
// they fly through the barrier and the stores; every CTA lets the next launch
// start as soon as it has started.
//
// Measured against the form it replaced (a warp owning up to 4 whole rows,
// 16 loads in flight a lane, 109 registers, two CTAs of 8 warps an SM), same
// bits: K=2048 N=8192 5.25 -> 3.78 us a launch, K=8192 N=2048 5.1 -> 4.2 us,
// the 2048 -> 128256 head 42.9 -> 38.8 us; the early trigger alone is
// 4.3-4.5 -> 3.78 us of that at K=2048 N=8192.
#pragma once

#include <cstdint>

#include "ptx.cuh"

namespace cgpu {

constexpr int NPU_MAX_TENSORS = 8;
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

constexpr uint32_t NPU_GROUP_ROWS = 8;
constexpr size_t NPU_SMEM_MAX = 16 * 1024;

// the activation, then two [W][8] buffers of warp partials
inline size_t npumv_smem_bytes(uint32_t kp, int w)
{
	return (size_t)kp + (size_t)2 * w * NPU_GROUP_ROWS * sizeof(int);
}
static_assert(NPU_INLINE_WORDS * 16 + 2 * 16 * NPU_GROUP_ROWS * sizeof(int) <= NPU_SMEM_MAX,
	      "the largest K's activation and partials fit the shared memory asked for");

template <int W, int U, int AW>
__device__ __forceinline__ void npumv_body(const NpuParams &p, const uint4 *inl)
{
	extern __shared__ __align__(16) uint8_t npu_smem[];
	constexpr uint32_t G8 = NPU_GROUP_ROWS;
	const uint32_t nch = p.kp / 16;
	uint4 *act = reinterpret_cast<uint4 *>(npu_smem);
	int *part = reinterpret_cast<int *>(npu_smem + p.kp);     // [2][W][8]
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const uint32_t groups = (p.total_rows + G8 - 1) / G8;
	constexpr uint32_t PASS = 32u * W * U;                      // chunks a pass
	const uint32_t npass = (nch + PASS - 1) / PASS;

	// row j of group G: its tensor and its bytes (nullptr past the last row)
	auto row_of = [&](uint32_t r, uint32_t &t) {
		t = 0;
		while (t + 1 < p.ntensor && r >= p.t[t].row_end)
			t++;
		return r - (p.t[t].row_end - p.t[t].rows);
	};
	const int8_t *wr[G8];
	auto setup = [&](uint32_t G) {
#pragma unroll
		for (uint32_t j = 0; j < G8; j++) {
			const uint32_t r = G * G8 + j;
			uint32_t t;
			const uint32_t lr = row_of(r < p.total_rows ? r : 0, t);
			wr[j] = r < p.total_rows ? p.t[t].w + (uint64_t)lr * p.kp : nullptr;
		}
	};
	uint4 wv[G8][U];
	auto load = [&](uint32_t pass) {
#pragma unroll
		for (int u = 0; u < U; u++) {
			const uint32_t c = pass * PASS + (uint32_t)(u * 32 * W + warp * 32 + lane);
#pragma unroll
			for (uint32_t j = 0; j < G8; j++)
				wv[j][u] = (wr[j] && c < nch) ? ldg_stream((const uint8_t *)wr[j] + c * 16)
							     : make_uint4(0, 0, 0, 0);
		}
	};
	// thread j < 8: its row's output and scale, loaded ahead of the sums
	auto out_of = [&](uint32_t G, float *&yp, float &sc) {
		const uint32_t r = G * G8 + threadIdx.x;
		yp = nullptr;
		sc = 0.0f;
		if (threadIdx.x < G8 && r < p.total_rows) {
			uint32_t t;
			const uint32_t lr = row_of(r, t);
			yp = p.t[t].y + lr;
			sc = p.t[t].scale[lr];
		}
	};

	pdl_launch_dependents();
	// the first group's first pass goes now: weights never depend on the
	// kernel before this one
	uint32_t G = blockIdx.x;
	float *yp = nullptr;
	float sc = 0.0f;
	if (G < groups) {
		setup(G);
		load(0);
		out_of(G, yp, sc);
	}
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

	for (uint32_t i = 0; G < groups; i++, G += gridDim.x) {
		int acc[G8];
#pragma unroll
		for (uint32_t j = 0; j < G8; j++)
			acc[j] = 0;
		for (uint32_t ps = 0; ps < npass; ps++) {
			if (ps)
				load(ps);
#pragma unroll
			for (int u = 0; u < U; u++) {
				const uint32_t c = ps * PASS + (uint32_t)(u * 32 * W + warp * 32 + lane);
				if (c < nch) {
					const uint4 a = act[c];
#pragma unroll
					for (uint32_t j = 0; j < G8; j++) {
						acc[j] = dp4a_s(wv[j][u].x, a.x, acc[j]);
						acc[j] = dp4a_s(wv[j][u].y, a.y, acc[j]);
						acc[j] = dp4a_s(wv[j][u].z, a.z, acc[j]);
						acc[j] = dp4a_s(wv[j][u].w, a.w, acc[j]);
					}
				}
			}
		}
		// the next group's first pass in flight before the sums
		const uint32_t Gn = G + gridDim.x;
		float *yp_n = nullptr;
		float sc_n = 0.0f;
		if (Gn < groups) {
			setup(Gn);
			load(0);
			out_of(Gn, yp_n, sc_n);
		}
		int *pb = part + (i & 1) * W * G8;
#pragma unroll
		for (uint32_t j = 0; j < G8; j++) {
			const int s = __reduce_add_sync(0xffffffffu, acc[j]);
			if ((uint32_t)lane == j)
				pb[warp * G8 + j] = s;
		}
		named_barrier(1, W * 32);
		if (yp) {
			int s = 0;
#pragma unroll
			for (int w = 0; w < W; w++)
				s += pb[w * G8 + threadIdx.x];
			*yp = __fmul_rn(__fmul_rn(__int2float_rn(s), d1), sc);
		}
		yp = yp_n;
		sc = sc_n;
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

template <int W, int U>
__global__ void __launch_bounds__(W * 32)
npumv_kernel(const __grid_constant__ NpuParams p)
{
	npumv_body<W, U, 0>(p, nullptr);
}

template <int W, int U, int AW>
__global__ void __launch_bounds__(W * 32)
npumv_inline_kernel(const __grid_constant__ NpuInline<AW> a)
{
	npumv_body<W, U, AW>(a.p, a.act);
}

} // namespace cgpu
