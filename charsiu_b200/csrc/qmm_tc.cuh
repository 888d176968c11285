// SPDX-License-Identifier: GPL-2.0-or-later
// The batched block-quant matvec on the tensor cores: m activations against
// a q8_0 tensor, y[a][n] bit-identical to charsiu's gguf_matvec of each
// activation (reference src/gguf.c:1098-1107, 1149-1171).
//
// One tcgen05.mma kind::i8 with K = 32 is exactly one GGML block: for block b
// it gives t[n][a] = sum_j q_w[n][b][j] * q_a[a][b][j] for a 128-row weight
// tile (the MMA's M: 16 eight-row groups) and NA activations (its N) into
// tensor memory. The epilogue then does what the reference does per block,
//     s[n][a] = s[n][a] + (d_w[n][b] * d_a[a][b]) * (float)t[n][a]
// in block order, so the fp32 sums are the reference's exactly. The MMA
// cannot accumulate across blocks (each block has its own scales); it writes
// a fresh int32 tile per block into one of two tensor-memory buffers while
// the epilogue drains the other.
//
// Warp roles: warp 0 lane 0 issues the single-destination bulk copies of one
// K segment (16 blocks) a stage -- the 16 groups' weight segments as they lie
// in the device layout (layout.h), already MMA core matrices, and the packed
// activation tile (qmm_pack_kernel) -- into a double-buffered stage; warp 1
// owns tensor memory and lane 0 issues the MMAs; 4 * EP epilogue warps (a
// lane quarter each, EP column slices of 32 when NA = 64) read the int32
// tiles with tcgen05.ld and accumulate. Every wait is bounded.
#pragma once

#include "layout.h"
#include "ptx.cuh"
#include "tcgen05.cuh"

namespace cgpu {

constexpr int QMM_TILE_GROUPS = 16;                       // 128 weight rows
constexpr uint32_t QMM_WSTAGE = QMM_TILE_GROUPS * MAX_SEG_BYTES;   // 69632

// The packed activation tile of a NA-row slab of activations, per K segment:
// quants [16 blocks][2 chunks][NA rows][16 B] then deltas [16 blocks][NA] f32.
// Rows past m and blocks past nb are zero.
__host__ __device__ constexpr uint32_t qmm_act_seg_bytes(uint32_t na)
{
	return SB * 2 * na * 16 + SB * na * 4;
}

__host__ inline size_t qmm_smem_bytes(uint32_t na)
{
	return 2 * ((size_t)QMM_WSTAGE + qmm_act_seg_bytes(na)) + 16 * sizeof(uint64_t) + 16;
}

// q int8 [m][nb*32], d f32 [m][nb] -> packed [m tiles][nseg][qmm_act_seg_bytes]
// One thread per 16-byte quant chunk or per delta.
__global__ void qmm_pack_kernel(const int8_t *__restrict__ q, const float *__restrict__ d,
				uint32_t m, uint32_t nb, uint32_t na, uint8_t *__restrict__ out)
{
	const uint32_t nseg = nsegments(nb), mt = (m + na - 1) / na;
	const uint64_t per_seg = (uint64_t)SB * 2 * na + (uint64_t)SB * na;   // work items
	const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
	if (idx >= (uint64_t)mt * nseg * per_seg)
		return;
	const uint32_t tile = (uint32_t)(idx / (nseg * per_seg));
	const uint64_t rem = idx % (nseg * per_seg);
	const uint32_t seg = (uint32_t)(rem / per_seg), w = (uint32_t)(rem % per_seg);
	uint8_t *base = out + ((uint64_t)tile * nseg + seg) * qmm_act_seg_bytes(na);
	if (w < (uint32_t)SB * 2 * na) {
		const uint32_t bi = w / (2 * na), c = (w / na) % 2, row = w % na;
		const uint32_t a = tile * na + row, blk = seg * SB + bi;
		uint4 v = make_uint4(0, 0, 0, 0);
		if (a < m && blk < nb)
			v = *reinterpret_cast<const uint4 *>(q + ((uint64_t)a * nb + blk) * 32 + c * 16);
		*reinterpret_cast<uint4 *>(base + ((bi * 2 + c) * na + row) * 16) = v;
	} else {
		const uint32_t w2 = w - SB * 2 * na, bi = w2 / na, row = w2 % na;
		const uint32_t a = tile * na + row, blk = seg * SB + bi;
		reinterpret_cast<float *>(base + SB * 2 * na * 16)[bi * na + row] =
			(a < m && blk < nb) ? d[(uint64_t)a * nb + blk] : 0.0f;
	}
}

struct QmmParams {
	const uint8_t *w;          // the tensor's device layout (q8_0)
	const uint8_t *act;        // qmm_pack_kernel output
	float *y;                  // y[a][rows]
	uint32_t rows, groups, nb, m;
	int *err;
};

template <int NA>
__global__ void __launch_bounds__((2 + 4 * (NA > 32 ? NA / 32 : 1)) * 32, 1)
qmm_tc_kernel(const __grid_constant__ QmmParams p)
{
	constexpr int EP = NA > 32 ? NA / 32 : 1;          // column slices
	constexpr int EC = NA / EP;                        // columns a slice
	constexpr uint32_t ASEG = qmm_act_seg_bytes(NA);
	extern __shared__ __align__(128) uint8_t smem[];
	auto stage_w = [&](uint32_t st) { return smem + st * QMM_WSTAGE; };
	auto stage_a = [&](uint32_t st) { return smem + 2 * QMM_WSTAGE + st * ASEG; };
	uint64_t *bars = reinterpret_cast<uint64_t *>(smem + 2 * (QMM_WSTAGE + ASEG));
	uint64_t *full = bars, *freeb = bars + 2, *mma_done = bars + 4, *tfree = bars + 6;
	uint32_t *taddr_s = reinterpret_cast<uint32_t *>(bars + 8);

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const uint32_t g0 = blockIdx.x * QMM_TILE_GROUPS, a0 = blockIdx.y * NA;
	const uint32_t nb = p.nb, nseg = nsegments(nb);
	const uint32_t tgroups = min((uint32_t)QMM_TILE_GROUPS, p.groups - g0);
	const uint8_t *act = p.act + (uint64_t)blockIdx.y * nseg * ASEG;

	if (warp == 1) {
		tmem_alloc(taddr_s, 2 * NA < 32 ? 32 : 2 * NA);
		tmem_relinquish();
	}
	if (threadIdx.x == 0) {
		for (int i = 0; i < 2; i++) {
			mbar_init(&full[i], 1);
			mbar_init(&freeb[i], 1 + 4 * EP);
			mbar_init(&mma_done[i], 1);
			mbar_init(&tfree[i], 4 * EP);
		}
		fence_mbar_init();
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t taddr = *taddr_s;

	if (warp == 0) {
		// ---- producer ------------------------------------------------------
		if (lane == 0) {
			for (uint32_t s = 0; s < nseg; s++) {
				const uint32_t st = s & 1, sb = seg_blocks(nb, s);
				if (s >= 2 && !mbar_wait_bounded(&freeb[st], ((s >> 1) - 1) & 1, WAIT_LIMIT_NS)) {
					*(volatile int *)p.err = 5;
					break;
				}
				const uint32_t wbytes = sb * block_group_bytes(TYPE_Q8_0);
				mbar_arrive_expect_tx(&full[st], tgroups * wbytes + ASEG);
				for (uint32_t g = 0; g < tgroups; g++)
					bulk_g2s(stage_w(st) + g * MAX_SEG_BYTES,
						 p.w + (uint64_t)(g0 + g) * group_bytes(TYPE_Q8_0, nb) +
							 seg_offset(TYPE_Q8_0, s),
						 wbytes, &full[st]);
				bulk_g2s(stage_a(st), act + (uint64_t)s * ASEG, ASEG, &full[st]);
			}
		}
	} else if (warp == 1) {
		// ---- MMA issuer ------------------------------------------------------
		if (lane == 0) {
			constexpr uint32_t idesc = idesc_i8(128, NA);
			bool ok = true;
			for (uint32_t s = 0; s < nseg && ok; s++) {
				const uint32_t st = s & 1, sb = seg_blocks(nb, s);
				if (!mbar_wait_bounded(&full[st], (s >> 1) & 1, WAIT_LIMIT_NS)) {
					*(volatile int *)p.err = 6;
					break;
				}
				tc_fence_after();
				for (uint32_t bi = 0; bi < sb; bi++) {
					const uint32_t j = s * SB + bi, buf = j & 1;
					if (j >= 2 && !mbar_wait_bounded(&tfree[buf], ((j >> 1) - 1) & 1,
									 WAIT_LIMIT_NS)) {
						*(volatile int *)p.err = 7;
						ok = false;
						break;
					}
					tc_fence_after();
					const uint64_t ad = smem_desc_k_nosw(stage_w(st) + bi * RG * 32, RG * 16,
									     MAX_SEG_BYTES);
					const uint64_t bd = smem_desc_k_nosw(stage_a(st) + bi * 2 * NA * 16,
									     NA * 16, 128);
					mma_i8(taddr + buf * NA, ad, bd, idesc, false);
					mma_commit(&mma_done[buf]);
				}
				mma_commit(&freeb[st]);
			}
		}
	} else {
		// ---- epilogue: TMEM lane quarter q, column slice e -------------------
		const int ew = warp - 2, q = warp % 4, e = ew / 4;
		const uint32_t r = q * 32 + lane;                  // row of the tile
		const uint32_t grp = r / RG, rr = r % RG;
		float acc[EC];
#pragma unroll
		for (int c = 0; c < EC; c++)
			acc[c] = 0.0f;
		bool ok = true;
		for (uint32_t s = 0; s < nseg && ok; s++) {
			const uint32_t st = s & 1, sb = seg_blocks(nb, s);
			if (!mbar_wait_bounded(&full[st], (s >> 1) & 1, WAIT_LIMIT_NS)) {
				if (lane == 0)
					*(volatile int *)p.err = 8;
				break;
			}
			const uint16_t *dl = reinterpret_cast<const uint16_t *>(
				stage_w(st) + grp * MAX_SEG_BYTES + sb * RG * 32);
			const float *da = reinterpret_cast<const float *>(stage_a(st) + SB * 2 * NA * 16);
			for (uint32_t bi = 0; bi < sb; bi++) {
				const uint32_t j = s * SB + bi, buf = j & 1;
				if (!mbar_wait_bounded(&mma_done[buf], (j >> 1) & 1, WAIT_LIMIT_NS)) {
					if (lane == 0)
						*(volatile int *)p.err = 9;
					ok = false;
					break;
				}
				tc_fence_after();
				uint32_t t[EC];
#pragma unroll
				for (int c = 0; c < EC; c += 16)
					tmem_ld16(taddr + ((uint32_t)(q * 32) << 16) + buf * NA + e * EC + c,
						  *reinterpret_cast<uint32_t(*)[16]>(&t[c]));
				tmem_wait_ld();
				tc_fence_before();
				__syncwarp();
				if (lane == 0)
					mbar_arrive(&tfree[buf]);
				const float dw = half_bits_to_float(dl[bi * RG + rr]);
				const float *dab = da + bi * NA + e * EC;
#pragma unroll
				for (int c = 0; c < EC; c++)
					acc[c] = __fadd_rn(acc[c], __fmul_rn(__fmul_rn(dw, dab[c]),
									     small_int_to_float((int32_t)t[c])));
			}
			__syncwarp();
			if (lane == 0)
				mbar_arrive(&freeb[st]);
		}
		const uint32_t row = g0 * RG + r;
		if (ok && row < p.rows) {
#pragma unroll
			for (int c = 0; c < EC; c++) {
				const uint32_t a = a0 + e * EC + c;
				if (a < p.m)
					p.y[(uint64_t)a * p.rows + row] = acc[c];
			}
		}
	}
	tc_fence_before();
	__syncthreads();
	if (warp == 1)
		tmem_dealloc(taddr, 2 * NA < 32 ? 32 : 2 * NA);
}

} // namespace cgpu
