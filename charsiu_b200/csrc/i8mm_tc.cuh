// SPDX-License-Identifier: GPL-2.0-or-later
// The int8 matmul with the NPU's output stage on the tensor cores, for M > 1
// (batched decode, prefill): tcgen05.mma kind::i8, int32 accumulator in
// tensor memory. Byte-exact against cpu_reference (tools/charsiu_matmul.c:41-81)
// by the same arithmetic as i8mm_simt_body (aux_kernels.cuh): signed
// operands a ^ 0x80 and w ^ 0x80, zero points folded in afterwards, the
// reference's float requant.
//
// A CTA owns 128 rows of a (the MMA's M) and NT rows of w (its N). K goes
// through shared memory in chunks of I8TC_KC bytes, zero-padded, laid out as
// K-major no-swizzle core matrices ([K step][16-byte chunk][row][16 B]); one
// thread issues the chunk's K = 32 MMAs, accumulating into tensor memory, and
// commits them to an mbarrier that every thread waits on (bounded) before the
// chunk's shared memory is refilled. Then 4 warps read their 32 accumulator
// lanes each with tcgen05.ld and run the output stage.
#pragma once

#include "aux_kernels.cuh"
#include "tcgen05.cuh"

namespace cgpu {

constexpr int I8TC_M = 128;
constexpr int I8TC_KC = 128;

template <int NT>
__global__ void __launch_bounds__(128) i8mm_tc_kernel(const __grid_constant__ I8Params p, int *err)
{
	__shared__ __align__(128) uint8_t As[I8TC_KC * I8TC_M];
	__shared__ __align__(128) uint8_t Bs[I8TC_KC * NT];
	__shared__ int32_t sa[I8TC_M], sw[NT];
	__shared__ __align__(8) uint64_t done;
	__shared__ uint32_t taddr_s;

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const uint32_t m0 = blockIdx.y * I8TC_M, n0 = blockIdx.x * NT;
	const uint32_t kpad = (p.k + 31) / 32 * 32;

	if (warp == 0) {
		tmem_alloc(&taddr_s, NT < 32 ? 32 : NT);
		tmem_relinquish();
	}
	if (threadIdx.x == 0) {
		mbar_init(&done, 1);
		fence_mbar_init();
	}
	// sum of the signed bytes of each row of a and of w, for the zero points
	{
		const uint32_t t = threadIdx.x;
		int s = 0;
		if (m0 + t < p.m)
			for (uint32_t k = 0; k < p.k; k++)
				s += (int8_t)(p.a[(uint64_t)(m0 + t) * p.k + k] ^ 0x80);
		sa[t] = s;
		for (uint32_t c = t; c < (uint32_t)NT; c += blockDim.x) {
			int v = 0;
			if (n0 + c < p.n)
				for (uint32_t k = 0; k < p.k; k++)
					v += (int8_t)(p.w[(uint64_t)(n0 + c) * p.k + k] ^ 0x80);
			sw[c] = v;
		}
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t taddr = taddr_s;
	bool ok = true;

	for (uint32_t k0 = 0, chunk = 0; k0 < kpad; k0 += I8TC_KC, chunk++) {
		const uint32_t kc = min((uint32_t)I8TC_KC, kpad - k0);
		// operands as core matrices: byte (row, kk) at
		// (kk / 32) * (2 * R * 16) + ((kk / 16) & 1) * (R * 16) + row * 16 + kk % 16
		for (uint32_t i = threadIdx.x; i < I8TC_M * kc; i += blockDim.x) {
			const uint32_t row = i / kc, kk = i % kc, gk = k0 + kk;
			const uint8_t v = (m0 + row < p.m && gk < p.k)
				? (uint8_t)(p.a[(uint64_t)(m0 + row) * p.k + gk] ^ 0x80) : 0;
			As[(kk / 32) * (2 * I8TC_M * 16) + ((kk / 16) & 1) * (I8TC_M * 16) + row * 16 +
			   kk % 16] = v;
		}
		for (uint32_t i = threadIdx.x; i < (uint32_t)NT * kc; i += blockDim.x) {
			const uint32_t row = i / kc, kk = i % kc, gk = k0 + kk;
			const uint8_t v = (n0 + row < p.n && gk < p.k)
				? (uint8_t)(p.w[(uint64_t)(n0 + row) * p.k + gk] ^ 0x80) : 0;
			Bs[(kk / 32) * (2 * NT * 16) + ((kk / 16) & 1) * (NT * 16) + row * 16 + kk % 16] = v;
		}
		fence_proxy_async_smem();
		__syncthreads();
		if (threadIdx.x == 0) {
			tc_fence_after();
			for (uint32_t s = 0; s < kc / 32; s++) {
				const uint64_t ad = smem_desc_k_nosw(As + s * (2 * I8TC_M * 16), I8TC_M * 16, 128);
				const uint64_t bd = smem_desc_k_nosw(Bs + s * (2 * NT * 16), NT * 16, 128);
				mma_i8(taddr, ad, bd, idesc_i8(I8TC_M, NT), k0 != 0 || s != 0);
			}
			mma_commit(&done);
		}
		if (!mbar_wait_bounded(&done, chunk & 1, WAIT_LIMIT_NS)) {
			if (threadIdx.x == 0)
				*(volatile int *)err = 4;
			ok = false;
			break;
		}
	}
	tc_fence_after();

	if (ok) {
		const uint32_t row = m0 + warp * 32 + lane;
		const int64_t ca = 128 - p.zp_a, cw = 128 - p.zp_w;
#pragma unroll
		for (int c = 0; c < NT; c += 16) {
			uint32_t r[16];
			tmem_ld16(taddr + ((uint32_t)(warp * 32) << 16) + c, r);
			tmem_wait_ld();
			if (row < p.m) {
				// 16 columns of one row: one 16-byte store when they are all
				// there and aligned (out may be mapped host memory, where a
				// byte store is a bus transaction of its own)
				uint32_t pk[4] = {0, 0, 0, 0};
#pragma unroll
				for (int j = 0; j < 16; j++) {
					const uint32_t col = n0 + c + j;
					if (col < p.n) {
						const int64_t total = (int64_t)p.bias[col] + (int32_t)r[j] +
							cw * sa[warp * 32 + lane] + ca * sw[c + j] +
							(int64_t)p.k * ca * cw;
						const int8_t o = output_stage(total, p.mult, p.zp_out);
						pk[j >> 2] |= (uint32_t)(uint8_t)o << (8 * (j & 3));
					}
				}
				const uint64_t o0 = (uint64_t)row * p.n + n0 + c;
				if (n0 + c + 16 <= p.n && (o0 & 15) == 0) {
					*reinterpret_cast<uint4 *>(p.out + o0) =
						make_uint4(pk[0], pk[1], pk[2], pk[3]);
				} else {
#pragma unroll
					for (int j = 0; j < 16; j++)
						if (n0 + c + j < p.n)
							p.out[o0 + j] = (int8_t)(pk[j >> 2] >> (8 * (j & 3)));
				}
			}
		}
	}
	tc_fence_before();
	__syncthreads();
	if (warp == 0)
		tmem_dealloc(taddr, NT < 32 ? 32 : NT);
	if (p.done_flag)
		i8_raise_flag(p.done_count, p.done_flag, p.seq);
}

} // namespace cgpu
