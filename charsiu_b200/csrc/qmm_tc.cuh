// SPDX-License-Identifier: GPL-2.0-or-later
// The batched block-quant matvec on the tensor cores: m activations against
// up to eight q8_0 tensors of one K, y[a][n] bit-identical to charsiu's
// gguf_matvec of each activation (reference src/gguf.c:1098-1107, 1149-1171).
//
// One tcgen05.mma kind::i8 with K = 32 is exactly one GGML block: for block b
// it gives t[n][a] = sum_j q_w[n][b][j] * q_a[a][b][j] for a 128-row weight
// tile (the MMA's M: 16 eight-row groups) and NA activations (its N) into
// tensor memory. The epilogue then does what the reference does per block,
//     s[n][a] = s[n][a] + (d_w[n][b] * d_a[a][b]) * (float)t[n][a]
// in block order, so the fp32 sums are the reference's exactly. The MMA
// cannot accumulate across blocks (each block has its own scales); it writes
// a fresh int32 tile per block. Tiles are grouped in CHUNKS of blocks (a
// whole 16-block segment at 16 activations, half of one at 32), one commit a
// chunk, into two chunk buffers of tensor memory, so the epilogue drains one
// chunk while the MMAs fill the other.
//
// Work units are (128-row tile of one tensor, NA activations, a slice of EC
// of those activations); a persistent grid deals them round robin, slice and
// activation tile fastest so the CTAs sharing a weight tile run together (the
// second and later reads of it hit L2). With EC < NA each CTA still issues
// the whole NA-wide MMA (the tensor pipe is nearly idle here) and its
// epilogue takes only its slice: two or four times the units, for launches
// too small to fill the SMs otherwise. Warp
// roles: warp 0 lane 0 issues the single-destination bulk copies of one K
// segment (16 blocks) a stage -- the tile's 16 groups' weight segments as
// they lie in the device layout (layout.h), already MMA core matrices, and
// the activation tile (two tiled tensor copies from q and d) -- into a double-buffered
// stage; warp 1 owns tensor memory and lane 0 issues the MMAs; EW = 4 * EC/8
// epilogue warps (a tensor-memory lane quarter and 8 activations each; four
// warps of 4 activations for a 4-wide slice) read
// the int32 tiles with tcgen05.ld and accumulate: four blocks a read, their
// products first (independent, so they overlap), then the four in-order sums.
// Every step uses the packed fp32x2 operations (two columns an instruction,
// each lane rounded as the scalar operation rounds).
//
// PRE: the tensor memory of every block slot holds 0x4b400000 before its MMA,
// which then accumulates onto it, so the int32 comes out as the bits of the
// float 1.5 * 2^23 + t and the epilogue's int-to-float is one subtraction
// (|t| <= 32 * 127 * 128 < 2^22). The epilogue writes the constant back after
// each read. Every wait is bounded.
#pragma once

#include <cuda.h>              // CUtensorMap

#include "layout.h"
#include "ptx.cuh"
#include "tcgen05.cuh"

namespace cgpu {

constexpr int QMM_TILE_GROUPS = 16;                       // 128 weight rows
constexpr uint32_t QMM_WSTAGE = QMM_TILE_GROUPS * MAX_SEG_BYTES;   // 69632
// Blocks a commit and chunk buffers: two buffers of 256 / NA blocks, the 512
// tensor-memory columns. One MMA of this shape (M = 128, K = 32, N <= 128)
// occupies the tensor pipe about 72 cycles whatever N is, and each commit
// the epilogue waits on and drains adds 200-280 cycles to the MMA chain, so
// the fewer chunks the better while the epilogue still overlaps the next
// chunk: 16 activations take a whole 16-block segment a commit, 32 take
// half of one. (Four buffers of four blocks: the 1B step at M = 16 / 32 / 64
// 1.206 / 1.299 / 1.594 ms, against 0.908 / 1.043 / 1.372 this way.) The
// epilogue reads a chunk four blocks at a time.
__host__ __device__ constexpr int qmm_chunk(int na)
{
	return 256 / na;
}
__host__ __device__ constexpr int qmm_tbufs(int)
{
	return 2;
}
constexpr int QMM_SUB = 4;                                // blocks an epilogue read
constexpr int QMM_MAX_TENSORS = 8;

// The staged activation tile of a NA-row slab of activations, per K segment:
// quants [16 blocks][2 chunks][NA rows][16 B] (MMA core matrices) then deltas
// [NA rows][16 blocks] f32. Rows past m and blocks past nb are zero. Two tiled
// tensor copies stage it straight from q and d (q viewed as [16-byte
// chunks][rows][16 B], a box of 32 chunks x NA rows; d as [rows][blocks], a
// box of NA x 16); where those cannot be described (q or d not 16-byte
// aligned, or a row of d not a multiple of 16 bytes), qmm_pack_kernel lays
// the same bytes out in global memory first and one bulk copy a stage
// brings them in.
__host__ __device__ constexpr uint32_t qmm_act_seg_bytes(uint32_t na)
{
	return SB * 2 * na * 16 + SB * na * 4;
}

constexpr int QMM_EPI_COLS = 8;            // activations (columns) an epilogue warp owns

// An epilogue warp's private copy of one segment's scales: the d_w of its 32
// rows (4 groups x 16 blocks x 8 rows fp16) and the d_a of its 8 activations
// (16 blocks x 8 fp32). Taken when the segment lands, so the stage can be
// refilled as soon as the MMAs are done with it.
constexpr uint32_t QMM_PRIV_DW = 4 * SB * RG * 2;                       // 1024
constexpr uint32_t QMM_PRIV_BYTES = QMM_PRIV_DW + SB * QMM_EPI_COLS * 4;  // 1536

__host__ __device__ constexpr uint32_t qmm_bar_bytes()
{
	return 24 * sizeof(uint64_t) + 16;
}

// epilogue warps: four (one a tensor-memory lane quarter) for each 8
// activations of a unit's slice; a 4-wide slice takes four warps of 4
__host__ __device__ constexpr int qmm_epi_warps(int ec)
{
	return 4 * (ec < QMM_EPI_COLS ? 1 : ec / QMM_EPI_COLS);
}

__host__ inline size_t qmm_smem_bytes(uint32_t na, uint32_t ec)
{
	return 2 * ((size_t)QMM_WSTAGE + qmm_act_seg_bytes(na)) + qmm_bar_bytes() +
	       (size_t)qmm_epi_warps((int)ec) * QMM_PRIV_BYTES;
}

__host__ __device__ constexpr int qmm_threads(int ec)
{
	return (2 + qmm_epi_warps(ec)) * 32;
}

// tensor-memory columns: qmm_tbufs chunk buffers of qmm_chunk blocks of NA columns
__host__ __device__ constexpr uint32_t qmm_tmem_cols(int na)
{
	return qmm_tbufs(na) * qmm_chunk(na) * na;
}

// q int8 [m][nb*32], d f32 [m][nb] -> packed [m tiles][nseg][qmm_act_seg_bytes]
// One thread per 16-byte quant chunk or per delta.
__global__ void qmm_pack_kernel(const int8_t *__restrict__ q, const float *__restrict__ d,
				uint32_t m, uint32_t nb, uint32_t na, uint8_t *__restrict__ out)
{
	pdl_wait();                 // q and d may come from the kernel before
	pdl_launch_dependents();
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
		const uint32_t w2 = w - SB * 2 * na, row = w2 / SB, bi = w2 % SB;
		const uint32_t a = tile * na + row, blk = seg * SB + bi;
		reinterpret_cast<float *>(base + SB * 2 * na * 16)[row * SB + bi] =
			(a < m && blk < nb) ? d[(uint64_t)a * nb + blk] : 0.0f;
	}
}

struct QmmTensor {
	const uint8_t *w;          // the tensor's device layout (q8_0)
	float *y;                  // y[a][rows]
	uint32_t rows, groups;
	uint32_t tile_end;         // running count of 128-row tiles through this tensor
	uint32_t pad_;
};

struct QmmParams {
	CUtensorMap qmap, dmap;    // q and d as the staged tile's two boxes (use_map)
	QmmTensor t[QMM_MAX_TENSORS];
	const uint8_t *act;        // qmm_pack_kernel output (!use_map)
	uint32_t use_map;
	uint32_t ntensor, tiles, atiles, nb, m;
	float one;                 // 1.0 (see the epilogue's sum)
	int *err;
};

// The batched matvec fused with its all-gather (every tensor column-split
// over `world` GPUs, one process a GPU), as qmv1.cuh does it for one
// activation: each y this rank computes is stored straight into every rank's
// full output y[r][tensor] ([m][ncols], at column row0 + row) over NVLink;
// once all this launch's CTAs are done, the last adds 1 to word signal_idx of
// every rank's sync array (a system-scope release). With wait_mult > 0 the
// producer first waits, before it copies the activations in, until its own
// word wait_idx reaches (epoch + wait_adj) * wait_mult, the epoch being word
// 0 (gather_epoch_kernel). world 0: no gather.
constexpr int QMM_MAX_RANKS = 8;

struct QmmGather {
	float *y[QMM_MAX_RANKS][QMM_MAX_TENSORS];
	uint32_t *sync[QMM_MAX_RANKS];
	uint32_t *cta_count;            // this GPU's: CTAs done, zero between launches
	uint32_t row0[QMM_MAX_TENSORS], ncols[QMM_MAX_TENSORS];
	uint32_t world, rank, signal_idx, wait_idx, wait_mult;
	int32_t wait_adj;
};

template <int NA, int EC, bool PRE>
__global__ void __launch_bounds__(qmm_threads(EC), 1)
qmm_tc_kernel(const __grid_constant__ QmmParams p, const __grid_constant__ QmmGather gth)
{
	constexpr int CW = EC < QMM_EPI_COLS ? EC : QMM_EPI_COLS;   // activations an epilogue warp
	constexpr int EW = qmm_epi_warps(EC);              // epilogue warps
	static_assert(CW == 8 || (CW == 4 && EC == 4), "epilogue warps of 8 activations, or one 4-wide slice");
	constexpr uint32_t SL = NA / EC;                   // slices a tile
	static_assert(NA % EC == 0 && EC % CW == 0 && (!PRE || EC == NA),
		      "slices of whole epilogue warps; PRE fills every column it reads");
	constexpr uint32_t ASEG = qmm_act_seg_bytes(NA);
	constexpr uint32_t NCOLS = qmm_tmem_cols(NA);
	constexpr uint32_t CH = qmm_chunk(NA), TB = qmm_tbufs(NA);   // blocks a chunk, buffers
	static_assert(CH % QMM_SUB == 0 && 4 + 2 * TB <= 24, "chunk of whole reads; barrier space");
	static_assert(NCOLS >= 32 && NCOLS <= 512 && (NCOLS & (NCOLS - 1)) == 0,
		      "tensor memory is allocated in powers of two, 32 to 512 columns");
	extern __shared__ __align__(128) uint8_t smem[];
	auto stage_w = [&](uint32_t st) { return smem + st * QMM_WSTAGE; };
	auto stage_a = [&](uint32_t st) { return smem + 2 * QMM_WSTAGE + st * ASEG; };
	uint64_t *bars = reinterpret_cast<uint64_t *>(smem + 2 * (QMM_WSTAGE + ASEG));
	uint64_t *full = bars, *freeb = bars + 2, *mma_done = bars + 4;
	uint64_t *tfree = mma_done + TB;
	uint32_t *taddr_s = reinterpret_cast<uint32_t *>(tfree + TB);
	uint8_t *priv_all = smem + 2 * (QMM_WSTAGE + ASEG) + qmm_bar_bytes();

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const uint32_t nb = p.nb, nseg = nsegments(nb);
	const uint32_t units = p.tiles * p.atiles * SL;

	if (warp == 1) {
		tmem_alloc(taddr_s, NCOLS);
		tmem_relinquish();
	}
	if (threadIdx.x == 0) {
		for (int i = 0; i < 2; i++) {
			mbar_init(&full[i], 1);
			mbar_init(&freeb[i], 1 + EW);
		}
		for (uint32_t i = 0; i < TB; i++) {
			mbar_init(&mma_done[i], 1);
			mbar_init(&tfree[i], EW);
		}
		fence_mbar_init();
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t taddr = *taddr_s;

	// the tensor and row tile of unit u
	auto locate = [&](uint32_t u, uint32_t &ti, uint32_t &tile) {
		const uint32_t rt = u / (p.atiles * SL);
		ti = 0;
		while (ti + 1 < p.ntensor && rt >= p.t[ti].tile_end)
			ti++;
		tile = rt - (ti ? p.t[ti - 1].tile_end : 0);
	};

	if (warp == 0) {
		// ---- producer ------------------------------------------------------
		if (lane == 0) {
			bool ok = true;
			uint32_t s_cnt = 0, waited_act = 0;
			for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
				uint32_t ti, tile;
				locate(u, ti, tile);
				const QmmTensor &T = p.t[ti];
				const uint32_t g0 = tile * QMM_TILE_GROUPS;
				const uint32_t tgroups = min((uint32_t)QMM_TILE_GROUPS, T.groups - g0);
				const uint32_t at = (u / SL) % p.atiles;
				const uint8_t *act = p.act + (uint64_t)at * nseg * ASEG;
				for (uint32_t s = 0; s < nseg; s++, s_cnt++) {
					const uint32_t st = s_cnt & 1, sb = seg_blocks(nb, s);
					if (s_cnt >= 2 &&
					    !mbar_wait_bounded(&freeb[st], ((s_cnt >> 1) - 1) & 1, WAIT_LIMIT_NS)) {
						*(volatile int *)p.err = 5;
						ok = false;
						break;
					}
					const uint32_t wbytes = sb * block_group_bytes(TYPE_Q8_0);
					mbar_arrive_expect_tx(&full[st], tgroups * wbytes + ASEG);
					for (uint32_t g = 0; g < tgroups; g++)
						bulk_g2s(stage_w(st) + g * MAX_SEG_BYTES,
							 T.w + (uint64_t)(g0 + g) * group_bytes(TYPE_Q8_0, nb) +
								 seg_offset(TYPE_Q8_0, s),
							 wbytes, &full[st]);
					if (!waited_act) {
						// weights never depend on the kernel before; the
						// packed activations do (and, fused with the
						// gather, the other ranks' part of them)
						pdl_wait();
						waited_act = 1;
						if (gth.wait_mult) {
							const uint32_t *syn = gth.sync[gth.rank];
							const uint32_t target =
								(uint32_t)((int32_t)ld_acquire_sys(&syn[0]) +
									   gth.wait_adj) * gth.wait_mult;
							const uint64_t w0 = globaltimer_ns();
							while ((int32_t)(ld_acquire_sys(&syn[gth.wait_idx]) -
									 target) < 0) {
								if (globaltimer_ns() - w0 > WAIT_LIMIT_NS) {
									*(volatile int *)p.err = 13;
									break;
								}
								__nanosleep(64);
							}
						}
					}
					if (p.use_map) {
						tma_load_3d(stage_a(st), &p.qmap, 0, (int)(at * NA),
							    (int)(s * 2 * SB), &full[st]);
						tma_load_2d(stage_a(st) + SB * 2 * NA * 16, &p.dmap,
							    (int)(s * SB), (int)(at * NA), &full[st]);
					} else {
						bulk_g2s(stage_a(st), act + (uint64_t)s * ASEG, ASEG, &full[st]);
					}
				}
			}
			// before leaving, let every copy issued land (already true unless
			// a wait above gave up)
			for (uint32_t i = s_cnt > 2 ? s_cnt - 2 : 0; i < s_cnt; i++)
				if (!mbar_wait_bounded(&full[i & 1], (i >> 1) & 1, WAIT_LIMIT_NS))
					*(volatile int *)p.err = 10;
		}
	} else if (warp == 1) {
		// ---- MMA issuer ------------------------------------------------------
		if (lane == 0) {
			constexpr uint32_t idesc = idesc_i8(128, NA);
			bool ok = true;
			uint32_t s_cnt = 0, c_cnt = 0;
			for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
				for (uint32_t s = 0; s < nseg && ok; s++, s_cnt++) {
					const uint32_t st = s_cnt & 1, sb = seg_blocks(nb, s);
					if (!mbar_wait_bounded(&full[st], (s_cnt >> 1) & 1, WAIT_LIMIT_NS)) {
						*(volatile int *)p.err = 6;
						ok = false;
						break;
					}
					tc_fence_after();
					for (uint32_t b0 = 0; b0 < sb; b0 += CH, c_cnt++) {
						const uint32_t buf = c_cnt % TB, use = c_cnt / TB;
						// PRE: the epilogue's first release of each buffer is
						// its fill with the constant
						if ((PRE || use >= 1) &&
						    !mbar_wait_bounded(&tfree[buf], (use - (PRE ? 0 : 1)) & 1,
								       WAIT_LIMIT_NS)) {
							*(volatile int *)p.err = 7;
							ok = false;
							break;
						}
						tc_fence_after();
						const uint32_t nblk = min(CH, sb - b0);
						for (uint32_t j = 0; j < nblk; j++) {
							const uint32_t bi = b0 + j;
							const uint64_t ad = smem_desc_k_nosw(
								stage_w(st) + bi * RG * 32, RG * 16, MAX_SEG_BYTES);
							const uint64_t bd = smem_desc_k_nosw(
								stage_a(st) + bi * 2 * NA * 16, NA * 16, 128);
							mma_i8(taddr + buf * CH * NA + j * NA, ad, bd, idesc,
							       PRE);
						}
						mma_commit(&mma_done[buf]);
					}
					if (ok)
						mma_commit(&freeb[st]);
				}
			}
			// the last chunk's MMAs must be done before tensor memory is freed
			if (c_cnt && !mbar_wait_bounded(&mma_done[(c_cnt - 1) % TB],
							((c_cnt - 1) / TB) & 1,
							WAIT_LIMIT_NS))
				*(volatile int *)p.err = 11;
		}
	} else {
		// ---- epilogue: TMEM lane quarter q, activations e*CW .. e*CW+CW-1 ----
		const int ew = warp - 2, q = warp % 4, e = ew / 4;
		const uint32_t r = q * 32 + lane;                  // row of the tile
		const uint32_t rr = r % RG;
		uint8_t *priv = priv_all + ew * QMM_PRIV_BYTES;
		const uint32_t lane_base = (uint32_t)(q * 32) << 16;
		bool ok = true;
		if (PRE) {
			for (uint32_t c = 0; c < NCOLS; c += NA)
				tmem_fill8(taddr + lane_base + c + e * CW, INT_FLOAT_MAGIC);
			tmem_wait_st();
			tc_fence_before();
			__syncwarp();
			if (lane == 0)
				for (uint32_t i = 0; i < TB; i++)
					mbar_arrive(&tfree[i]);
		}
		pdl_wait();                  // y may still be read by the kernel before
		pdl_launch_dependents();
		const uint64_t neg_bias = pack2(-INT_FLOAT_BIAS, -INT_FLOAT_BIAS);
		const uint64_t one2 = pack2(p.one, p.one);
		uint32_t s_cnt = 0, c_cnt = 0;
		for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
			uint32_t ti, tile;
			locate(u, ti, tile);
			const uint32_t cb = (u % SL) * EC + e * CW;   // this warp's first column of the tile
			uint64_t acc[CW / 2];           // column pairs, packed
#pragma unroll
			for (int c = 0; c < CW / 2; c++)
				acc[c] = 0;                 // +0.0f, +0.0f
			for (uint32_t s = 0; s < nseg && ok; s++, s_cnt++) {
				const uint32_t st = s_cnt & 1, sb = seg_blocks(nb, s);
				if (!mbar_wait_bounded(&full[st], (s_cnt >> 1) & 1, WAIT_LIMIT_NS)) {
					if (lane == 0)
						*(volatile int *)p.err = 8;
					ok = false;
					break;
				}
				// this warp's scales of the segment into its private copy, then
				// the stage is free as far as the epilogue goes: word w of a
				// group's d_w (16 bytes) is block w's 8 rows; lane L's d_a
				// word is block L/2, activations cb + 4*(L&1) ..
				{
					const uint32_t g0 = (uint32_t)q * 4;
#pragma unroll
					for (int h = 0; h < 2; h++) {
						const uint32_t idx = lane + 32 * h, gl = idx / SB, w = idx % SB;
						reinterpret_cast<uint4 *>(priv)[idx] =
							*reinterpret_cast<const uint4 *>(
								stage_w(st) + (g0 + gl) * MAX_SEG_BYTES +
								sb * RG * 32 + w * 16);
					}
					// (CW = 4: lane L < 16 copies block L's 4), transposed from
					// the stage's [row][block] order
					const uint32_t bi = CW == 8 ? lane >> 1 : lane, hf = CW == 8 ? lane & 1 : 0;
					if (CW == 8 || lane < SB) {
						const float *ds = reinterpret_cast<const float *>(
							stage_a(st) + SB * 2 * NA * 16) + (cb + 4 * hf) * SB + bi;
						reinterpret_cast<float4 *>(priv + QMM_PRIV_DW)[lane] =
							make_float4(ds[0], ds[SB], ds[2 * SB], ds[3 * SB]);
					}
				}
				__syncwarp();
				if (lane == 0)
					mbar_arrive(&freeb[st]);
				const uint16_t *dl = reinterpret_cast<const uint16_t *>(priv) + (lane / RG) * SB * RG;
				const float *da = reinterpret_cast<const float *>(priv + QMM_PRIV_DW);
				for (uint32_t c0 = 0; c0 < sb; c0 += CH, c_cnt++) {
					const uint32_t buf = c_cnt % TB, cblk = min(CH, sb - c0);
					if (!mbar_wait_bounded(&mma_done[buf], (c_cnt / TB) & 1, WAIT_LIMIT_NS)) {
						if (lane == 0)
							*(volatile int *)p.err = 9;
						ok = false;
						break;
					}
					tc_fence_after();
					for (uint32_t b0 = c0; b0 < c0 + cblk; b0 += QMM_SUB) {
						const uint32_t nblk = min((uint32_t)QMM_SUB, c0 + cblk - b0);
						// four blocks' tiles as packed float bits 1.5 * 2^23 + t
						static_assert(QMM_SUB == 4, "tmem_ld_chunk4 shape");
						uint64_t tp[QMM_SUB][CW / 2];
						const uint32_t col0 = taddr + lane_base + buf * CH * NA + (b0 - c0) * NA + cb;
						if constexpr (CW == 8) {
							if (nblk == QMM_SUB)
								tmem_ld_chunk4<!PRE>(col0, NA, tp);
							else
								for (int j = 0; j < (int)nblk; j++)
									tmem_ld_block<!PRE>(col0 + j * NA, tp[j]);
						} else {
							if (nblk == QMM_SUB)
								tmem_ld_chunk4_c4(col0, NA, tp);
							else
								for (int j = 0; j < (int)nblk; j++)
									tmem_ld_block_c4(col0 + j * NA, tp[j]);
						}
						if (PRE) {
#pragma unroll
							for (int j = 0; j < QMM_SUB; j++)
								if (j < (int)nblk)
									tmem_fill8(col0 + j * NA, INT_FLOAT_MAGIC);
							tmem_wait_st();
						}
						// the chunk's last read releases its buffer to the MMAs
						if (b0 + QMM_SUB >= c0 + cblk) {
							tc_fence_before();
							__syncwarp();
							if (lane == 0)
								mbar_arrive(&tfree[buf]);
						}

						// block j's products (d_w * d_a) * t, CW columns in pairs
						auto products = [&](int j, uint64_t (&pr)[CW / 2]) {
							const uint32_t bi = b0 + j;
							const float dw = half_bits_to_float(dl[bi * RG + rr]);
							const uint64_t dw2 = pack2(dw, dw);
							const ulonglong2 *da2 = reinterpret_cast<const ulonglong2 *>(da + bi * CW);
#pragma unroll
							for (int c4 = 0; c4 < CW / 4; c4++) {
								const ulonglong2 a = da2[c4];
								const uint64_t f0 = add2_rn(tp[j][2 * c4], neg_bias);
								const uint64_t f1 = add2_rn(tp[j][2 * c4 + 1], neg_bias);
								pr[2 * c4] = mul2_rn(mul2_rn(dw2, a.x), f0);
								pr[2 * c4 + 1] = mul2_rn(mul2_rn(dw2, a.y), f1);
							}
						};
						// s = s + product, block by block: fma(product, 1, s) with the
						// 1 from the kernel's parameters is the rounded add (a packed
						// add fed by the packed product would be contracted into one
						// rounding, unlike the reference's two)
						if (nblk == QMM_SUB) {
							uint64_t pr[QMM_SUB][CW / 2];
#pragma unroll
							for (int j = 0; j < QMM_SUB; j++)
								products(j, pr[j]);
#pragma unroll
							for (int j = 0; j < QMM_SUB; j++)
#pragma unroll
								for (int c = 0; c < CW / 2; c++)
									acc[c] = fma2_rn(pr[j][c], one2, acc[c]);
						} else {
							for (int j = 0; j < (int)nblk; j++) {
								uint64_t pr[CW / 2];
								products(j, pr);
#pragma unroll
								for (int c = 0; c < CW / 2; c++)
									acc[c] = fma2_rn(pr[c], one2, acc[c]);
							}
						}
					}
				}
				__syncwarp();      // the private copy is read until here
			}
			if (!ok)
				break;
			const QmmTensor &T = p.t[ti];
			const uint32_t row = tile * QMM_TILE_GROUPS * RG + r;
			const uint32_t a0 = ((u / SL) % p.atiles) * NA + cb;
			if (row < T.rows) {
#pragma unroll
				for (int c = 0; c < CW; c++) {
					const uint32_t a = a0 + c;
					const float v = c & 1 ? hi2(acc[c / 2]) : lo2(acc[c / 2]);
					if (a >= p.m)
						continue;
					if (gth.world) {
						for (uint32_t r = 0; r < gth.world; r++)
							gth.y[r][ti][(uint64_t)a * gth.ncols[ti] + gth.row0[ti] +
								     row] = v;
					} else {
						T.y[(uint64_t)a * T.rows + row] = v;
					}
				}
			}
		}
	}
	tc_fence_before();
	__syncthreads();
	if (warp == 1)
		tmem_dealloc(taddr, NCOLS);
	// every rank's stores of this CTA (peer ones included) reach thread 0
	// through the barrier and are released at device scope by its count; the
	// last CTA acquires them all and tells every rank with relaxed
	// system-scope adds after one system-scope acq_rel fence (a release
	// pattern, as the M = 1 gather's end)
	if (gth.world && threadIdx.x == 0 &&
	    atom_add_acq_rel_gpu(gth.cta_count, 1u) == gridDim.x - 1) {
		*gth.cta_count = 0;
		fence_acq_rel_sys();
		for (uint32_t r = 0; r < gth.world; r++)
			red_relaxed_sys_add(gth.sync[r] + gth.signal_idx, 1u);
	}
}

} // namespace cgpu
