// SPDX-License-Identifier: GPL-2.0-or-later
// The single-activation (M = 1) block-quant matvec: the decode hot path.
//
// Same arithmetic as qmv.cuh (bit-identical to charsiu's gguf_matvec,
// reference src/gguf.c:1061-1107, 1149-1171), organised for occupancy:
//
//   A CTA of W warps owns one 8-row group at a time (groups dealt round robin
//   over a persistent grid). The group's 16-block segments are split over the
//   W warps (segment s to warp s mod W, at most two a warp). Each warp loads its segment straight
//   into registers with 16-byte non-allocating global loads -- every load of
//   the segment issued before any arithmetic, and the first segment's issued
//   before griddepcontrol.wait, since weights do not depend on the previous
//   kernel -- and turns it into 16 blocks x 8 rows of independent fp32 terms
//   (d_w * d_a) * t in a shared term buffer.
//
//   One named barrier per group; then warp 0's lanes 0..7 add their row's
//   terms in block order (the only serial part, one fadd per block) and store
//   y, while the other warps already load the next group into the other term
//   buffer. (A dedicated summing warp fed by per-segment flags was measured
//   slower: its registers cost more occupancy than its overlap gained.)
//
// Shared memory is the activation plus two term buffers (10 KB at K = 2048,
// 26 KB at K = 8192), so several CTAs share an SM and their loads keep
// enough bytes in flight to cover HBM latency.
#pragma once

#include "layout.h"
#include "ptx.cuh"
#include "qmv.cuh"

namespace cgpu {

// (+16: the inline form copies the activation in whole 16-byte words)
inline size_t qmv1_smem_bytes(uint32_t nb)
{
	return (size_t)2 * nb * RG * sizeof(float) +
	       (size_t)nb * (32 + sizeof(float) + sizeof(int32_t)) + 16;
}

// The activation carried in the launch's own parameters (the direct host
// call): the [q | d] block of nb * 36 bytes, in 16-byte words. The launch
// brings it to the GPU with the kernel's arguments, so the call needs no copy
// and no copy-in kernel. AW words: 144 (K <= 2048), 576 (K <= 8192), 1008
// (K <= 14336); parameter space holds up to 32764 bytes.
template <int AW>
struct QmvInline {
	QmvParams p;
	uint4 act[AW];
};
constexpr int QMV_INLINE_MAX_WORDS = 1008;

// The matvec fused with its all-gather (a tensor column-split over `world`
// GPUs, one process a GPU): this rank computes its slab of rows and stores
// each y straight into every rank's full output over NVLink (peer stores),
// then, once all its CTAs are done, adds its number of 8-row groups to every
// rank's arrival counter for this launch (a system-scope release). A later launch that reads the
// gathered output first waits, on its own GPU, until its arrival counter
// shows every rank's groups for this token. sync words: [0] the token epoch
// (gather_epoch_kernel adds 1 at each token's start), [1 + k] the arrivals
// of launch k, monotonic: after token t it holds (t + 1) * groups of launch k.
constexpr int QMV_MAX_RANKS = 8;

struct QmvGather {
	float *y[QMV_MAX_RANKS][QMV_MAX_TENSORS];  // each rank's full output of each tensor
	uint32_t *sync[QMV_MAX_RANKS];              // each rank's sync words
	uint32_t *cta_count;                        // this GPU's: CTAs done, zero between launches
	uint32_t row0[QMV_MAX_TENSORS];             // this rank's first row of each tensor
	uint32_t world, rank;
	uint32_t signal_idx;                        // arrival word this launch adds to
	uint32_t wait_idx, wait_mult;               // wait for sync[wait_idx] >= (epoch + adj) * mult
	int32_t wait_adj;                           // (wait_mult 0: no wait)
};

// Launched with programmatic dependence, it lets the next launch start at
// once (that one's weights then stream in meanwhile) and adds to the epoch
// only once the launch before it -- whose CTAs read the epoch -- is done.
__global__ void gather_epoch_kernel(uint32_t *sync_local)
{
	pdl_launch_dependents();
	pdl_wait();
	if (threadIdx.x == 0 && blockIdx.x == 0)
		sync_local[0] += 1;
}
static_assert(sizeof(QmvInline<QMV_INLINE_MAX_WORDS>) <= 32764, "kernel parameter space");

// One segment's raw bytes for this lane: step j covers blocks 4j..4j+3; lane
// l reads block p = l>>3, row r = l&7 (q8_0: its two 16-byte chunks; q4_0:
// its one) and that block-row's fp16 delta.
template <bool Q8>
struct SegRegs {
	uint4 w[SB / 4][Q8 ? 2 : 1];
	uint16_t dl[SB / 4];
};

template <bool Q8>
__device__ __forceinline__ void seg_load(SegRegs<Q8> &R, const uint8_t *seg, uint32_t sb, int lane)
{
	constexpr uint32_t QB = Q8 ? 32 : 16;
	const int p = lane >> 3, r = lane & 7;
#pragma unroll
	for (int j = 0; j < SB / 4; j++) {
		const uint32_t bl = min((uint32_t)(j * 4 + p), sb - 1);
		if ((uint32_t)j * 4 < sb) {
			const uint8_t *wp = seg + bl * RG * QB + r * 16;
			R.w[j][0] = ldg_stream(wp);
			if (Q8)
				R.w[j][Q8 ? 1 : 0] = ldg_stream(wp + RG * 16);
			R.dl[j] = ldg_stream_u16(seg + (size_t)sb * RG * QB + (bl * RG + r) * 2);
		}
	}
}

template <bool Q8>
__device__ __forceinline__ void seg_compute(const SegRegs<Q8> &R, uint32_t sb, uint32_t b0,
					    const int8_t *aq, const float *ad, const int32_t *asum,
					    int lane, float *tb)
{
	const int p = lane >> 3, r = lane & 7;
#pragma unroll
	for (int j = 0; j < SB / 4; j++) {
		const uint32_t bl = (uint32_t)(j * 4 + p);
		if ((uint32_t)j * 4 >= sb)
			break;
		if (bl >= sb)
			continue;
		const uint32_t blk = b0 + bl;
		const uint4 *ap = reinterpret_cast<const uint4 *>(aq + (size_t)blk * 32);
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
			t = t0 + t1 - 8 * asum[blk];
		}
		tb[blk * RG + r] = __fmul_rn(__fmul_rn(half_bits_to_float(R.dl[j]), ad[blk]),
					     __int2float_rn(t));
	}
}

// W warps a CTA; all tensors of one launch share one quant type (Q8). A warp
// handles segment warp of each group and, when TWO, also warp + W (so
// nseg <= W, or nseg <= 2W with TWO); both are loaded before either is
// computed.
template <int W, bool Q8, bool TWO, int AW>
__device__ __forceinline__ void qmv1_body(const QmvParams &p, const uint4 *inl,
					  const QmvGather *gth = nullptr)
{
	extern __shared__ __align__(128) uint8_t smem[];
	const uint32_t nb = p.nb;
	float *terms = reinterpret_cast<float *>(smem);
	int8_t *aq = reinterpret_cast<int8_t *>(terms + (size_t)2 * nb * RG);
	float *ad = reinterpret_cast<float *>(aq + (size_t)nb * 32);
	int32_t *asum = reinterpret_cast<int32_t *>(ad + nb);
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

	if (p.early_trigger)
		pdl_launch_dependents();
	// weights do not depend on the previous kernel: the first group's go now
	uint32_t G = blockIdx.x;
	if (G < p.total_groups)
		load(G);

	if (AW) {
		// [q | d] from parameter space to the same contiguous [aq | ad]
		if (p.done_flag && blockIdx.x == 0 && threadIdx.x == 0)
			*p.t_start = globaltimer_ns();
		uint4 *sa = reinterpret_cast<uint4 *>(aq);
		const uint32_t n16 = (nb * 36 + 15) / 16;
		for (uint32_t i = threadIdx.x; i < n16; i += blockDim.x)
			sa[i] = inl[i];
	}
	pdl_wait();
	if (gth && gth->wait_mult) {
		// the gathered input of this launch: every rank's part must be in
		if (threadIdx.x == 0) {
			const uint32_t *syn = gth->sync[gth->rank];
			const uint32_t target =
				(uint32_t)((int32_t)ld_acquire_sys(&syn[0]) + gth->wait_adj) * gth->wait_mult;
			const unsigned long long t0 = globaltimer_ns();
			while ((int32_t)(ld_acquire_sys(&syn[gth->wait_idx]) - target) < 0) {
				if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
					*(volatile int *)p.err = 12;
					break;
				}
				__nanosleep(64);
			}
		}
		__syncthreads();
	}
	if (!AW) {
		const uint4 *gq = reinterpret_cast<const uint4 *>(p.q);
		uint4 *sq = reinterpret_cast<uint4 *>(aq);
		for (uint32_t i = threadIdx.x; i < nb * 2; i += blockDim.x)
			sq[i] = gq[i];
		for (uint32_t i = threadIdx.x; i < nb; i += blockDim.x)
			ad[i] = p.d[i];
	}
	__syncthreads();
	if (!Q8) {
		for (uint32_t i = threadIdx.x; i < nb; i += blockDim.x) {
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
	if (!p.early_trigger)
		pdl_launch_dependents();

	for (uint32_t i = 0; G < p.total_groups; i++, G += gridDim.x) {
		uint32_t ti, lg;
		locate(G, ti, lg);
		float *tb = terms + (size_t)(i & 1) * nb * RG;
		if (i)
			load(G);
		if (s0 < nseg)
			seg_compute<Q8>(R0, seg_blocks(nb, s0), s0 * SB, aq, ad, asum, lane, tb);
		if (TWO && s1 < nseg)
			seg_compute<Q8>(R1, seg_blocks(nb, s1), s1 * SB, aq, ad, asum, lane, tb);
		named_barrier(1, W * 32);
		if (warp == 0 && lane < RG) {
			const float *t = tb + lane;
			float s = 0.0f;
#pragma unroll 16
			for (uint32_t b = 0; b < nb; b++)
				s = __fadd_rn(s, t[b * RG]);
			const uint32_t row = lg * RG + lane;
			if (row < p.t[ti].rows) {
				if (gth) {
					for (uint32_t r = 0; r < gth->world; r++)
						gth->y[r][ti][gth->row0[ti] + row] = s;
				} else {
					p.t[ti].y[row] = s;
				}
			}
		}
	}
	if (gth) {
		// this CTA's stores (peer ones included) reach thread 0 through the
		// barrier and are released at device scope by its count; the last CTA
		// acquires every CTA's, and one system-scope acq_rel fence then makes
		// its relaxed system-scope adds to every rank's arrival word a release
		// of all of them (a fence and a strong write: the memory model's
		// release pattern). Against a release add per rank after
		// __threadfence_system: the split head at 2 GPUs 26.7 -> 23.7 us, one
		// stream's column split 0.62 -> 0.42 ms a token; a system-scope
		// release in every CTA costs several microseconds.
		__syncthreads();
		if (threadIdx.x == 0 && atom_add_acq_rel_gpu(gth->cta_count, 1u) == gridDim.x - 1) {
			*gth->cta_count = 0;
			fence_acq_rel_sys();
			for (uint32_t r = 0; r < gth->world; r++)
				red_relaxed_sys_add(gth->sync[r] + gth->signal_idx, p.total_groups);
		}
	}
	if (p.done_flag) {
		// y is host memory. The barrier brings this CTA's stores to thread 0,
		// whose acq_rel count releases them at device scope; the last CTA's
		// count acquires every CTA's, and its system fence orders all of them
		// before the flag the host spins on. (A system fence in every thread
		// costs several microseconds a call; this costs one.)
		__syncthreads();
		if (threadIdx.x == 0 && atom_add_acq_rel_gpu(p.done_count, 1u) == gridDim.x - 1) {
			*p.done_count = 0;
			const unsigned long long t1 = globaltimer_ns();
			const unsigned long long dt = t1 - *(volatile const unsigned long long *)p.t_start;
			__threadfence_system();
			p.done_flag[1] = dt > 0xffffffffull ? 0xffffffffu : (uint32_t)dt;
			__threadfence_system();
			*(volatile uint32_t *)p.done_flag = p.seq;
		}
	}
}

template <int W, bool Q8, bool TWO>
__global__ void __launch_bounds__(W * 32)
qmv1_kernel(const __grid_constant__ QmvParams p)
{
	qmv1_body<W, Q8, TWO, 0>(p, nullptr);
}

template <int W, bool Q8, bool TWO>
__global__ void __launch_bounds__(W * 32)
qmv1_gather_kernel(const __grid_constant__ QmvParams p, const __grid_constant__ QmvGather gth)
{
	qmv1_body<W, Q8, TWO, 0>(p, nullptr, &gth);
}

template <int W, bool Q8, bool TWO, int AW>
__global__ void __launch_bounds__(W * 32)
qmv1_inline_kernel(const __grid_constant__ QmvInline<AW> a)
{
	qmv1_body<W, Q8, TWO, AW>(a.p, a.act);
}

} // namespace cgpu
