// SPDX-License-Identifier: GPL-2.0-or-later
// The smaller kernels: the load-time repack, the activation quantiser, the
// block-dot test hook, and the CUDA-core int8 matmul with the output stage.
#pragma once

#include "layout.h"
#include "ptx.cuh"

namespace cgpu {

// GGUF blocks -> the layout of layout.h. raw holds `nrows` rows of this GPU's
// slab starting at slab row `row0`; one thread per (row, block). The layout
// buffer was zeroed first, which is what the padding rows need.
__global__ void repack_kernel(const uint8_t *__restrict__ raw, uint32_t type, uint32_t nb,
			      uint32_t row0, uint32_t nrows, uint8_t *__restrict__ dst)
{
	const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
	if (idx >= (uint64_t)nrows * nb)
		return;
	const uint32_t rl = (uint32_t)(idx / nb), b = (uint32_t)(idx % nb);
	const uint32_t r = row0 + rl, g = r / RG, rr = r % RG;
	const uint32_t seg = b / SB, bi = b % SB, sb = seg_blocks(nb, seg);
	const uint32_t qb = quant_bytes(type), bsz = qb + 2;
	const uint8_t *src = raw + ((uint64_t)rl * nb + b) * bsz;
	uint8_t *segp = dst + (uint64_t)g * group_bytes(type, nb) + seg_offset(type, seg);
	uint8_t *dd = segp + (uint64_t)sb * RG * qb + ((uint64_t)bi * RG + rr) * 2;

	for (uint32_t j = 0; j < qb; j++)
		segp[quant_offset(type, bi, j / 16, rr) + j % 16] = src[2 + j];
	dd[0] = src[0];
	dd[1] = src[1];
}

// gguf_row_f32 of one row (reference src/gguf.c:1217-1256) read back out of
// the device layout: q8_0 d * q, q4_0 d * (nibble - 8), q6_K (d * scale) * q
// (deq_q6_K, src/gguf.c:457-479). The row index is read from device memory
// (*row); an index outside [0, rows) writes 1 to *err and leaves out alone.
// One thread an element.
__global__ void row_f32_kernel(const uint8_t *__restrict__ data, uint32_t type, uint64_t k,
			       uint32_t rows, const int32_t *__restrict__ row,
			       float *__restrict__ out, int *__restrict__ err)
{
	pdl_wait();
	const int32_t r = *row;
	const uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
	if (r < 0 || (uint32_t)r >= rows) {
		if (e == 0)
			*err = 1;
		return;
	}
	if (e >= k)
		return;
	if (type == TYPE_Q6_K) {
		const uint32_t nsb = (uint32_t)(k / 256), i = (uint32_t)(e / 256), w = (uint32_t)(e % 256);
		const uint8_t *wr = data + (uint64_t)r * q6k_row_bytes(nsb);
		const uint8_t *sb = wr + (size_t)i * 208;
		const uint32_t h = w / 128, kk = (w % 128) / 32, l = w % 32;
		const uint8_t lo = sb[h * 64 + (kk & 1) * 32 + l];
		const uint32_t nib = (kk & 2) ? lo >> 4 : lo & 0x0fu;
		const int q = (int)(nib | ((sb[128 + h * 32 + l] >> (2 * kk)) & 3u) << 4) - 32;
		const int8_t sc = (int8_t)sb[192 + h * 8 + l / 16 + 2 * kk];
		const uint16_t db = (uint16_t)(wr[(size_t)nsb * 208 + 2 * i] |
					       wr[(size_t)nsb * 208 + 2 * i + 1] << 8);
		out[e] = __fmul_rn(__fmul_rn(half_bits_to_float(db), (float)sc), (float)q);
		return;
	}
	const uint32_t nb = (uint32_t)(k / 32), b = (uint32_t)(e / 32), j = (uint32_t)(e % 32);
	const uint32_t g = (uint32_t)r / RG, rr = (uint32_t)r % RG;
	const uint32_t seg = b / SB, bi = b % SB, sbn = seg_blocks(nb, seg), qb = quant_bytes(type);
	const uint8_t *segp = data + (uint64_t)g * group_bytes(type, nb) + seg_offset(type, seg);
	const uint8_t *dp = segp + (uint64_t)sbn * RG * qb + ((uint64_t)bi * RG + rr) * 2;
	const float dd = half_bits_to_float((uint16_t)(dp[0] | dp[1] << 8));
	int q;
	if (type == TYPE_Q8_0) {
		q = (int8_t)segp[quant_offset(type, bi, j / 16, rr) + j % 16];
	} else {
		const uint8_t byte = segp[quant_offset(type, bi, 0, rr) + j % 16];
		q = (int)(j < 16 ? byte & 0x0f : byte >> 4) - 8;
	}
	out[e] = __fmul_rn(dd, (float)q);
}

// The integer block dots of rows [0, rows), read back out of the layout: the
// test hook that pins both the repack and the dot against dotq_*'s t.
__global__ void block_dots_kernel(const uint8_t *__restrict__ data, uint32_t type,
				  uint32_t rows, uint32_t nb, const int8_t *__restrict__ q,
				  int32_t *__restrict__ dots)
{
	const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
	if (idx >= (uint64_t)rows * nb)
		return;
	const uint32_t r = (uint32_t)(idx / nb), b = (uint32_t)(idx % nb);
	const uint32_t g = r / RG, rr = r % RG, seg = b / SB, bi = b % SB;
	const uint32_t qb = quant_bytes(type);
	const uint8_t *segp = data + (uint64_t)g * group_bytes(type, nb) + seg_offset(type, seg);
	const uint8_t *qp = segp + quant_offset(type, bi, 0, rr);
	const int8_t *x = q + (uint64_t)b * 32;
	int t = 0;

	(void)qb;
	if (type == TYPE_Q8_0) {
		for (int j = 0; j < 32; j++)
			t += (int)(int8_t)segp[quant_offset(type, bi, j / 16, rr) + j % 16] * x[j];
	} else {
		for (int j = 0; j < 16; j++) {
			t += ((qp[j] & 0x0f) - 8) * x[j];
			t += ((qp[j] >> 4) - 8) * x[j + 16];
		}
	}
	dots[idx] = t;
}

// charsiu_act_set (reference src/gguf.c:852-881) for m rows of k: one warp
// per 32-element block. amax is a max, so any reduction order gives the same
// float; d = amax / 127 and 1 / d are IEEE divisions; the quant is
// round-to-nearest-even of v * (1 / d), as lrintf.
__global__ void act_quantise_kernel(const float *__restrict__ x, uint32_t m, uint32_t k,
				    uint32_t nb, int8_t *__restrict__ q, float *__restrict__ d)
{
	const uint64_t w = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
	const int lane = threadIdx.x & 31;
	if (w >= (uint64_t)m * nb)
		return;
	const uint32_t row = (uint32_t)(w / nb), b = (uint32_t)(w % nb);
	const uint32_t i = b * 32 + lane;
	const float v = i < k ? x[(uint64_t)row * k + i] : 0.0f;
	float amax = fabsf(v);

	for (int o = 16; o; o >>= 1)
		amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
	const float dd = __fdiv_rn(amax, 127.0f);
	const float inv = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
	q[(uint64_t)row * nb * 32 + i] = (int8_t)__float2int_rn(__fmul_rn(v, inv));
	if (lane == 0)
		d[(uint64_t)row * nb + b] = dd;
}

// ---- the int8 matmul with the NPU's output stage -----------------------------
//
// acc = bias + sum_k (a - zp_a)(w - zp_w), a and w unsigned bytes. With
// a_s = a - 128 and w_s = w - 128 (signed bytes):
//   sum (a - zp_a)(w - zp_w) = sum a_s w_s + (128 - zp_w) sum a_s
//                              + (128 - zp_a) sum w_s + K (128 - zp_a)(128 - zp_w)
// the same zero-point folding the NPU's coefficient buffer does
// (reference src/job.c:298-303, 344).
//
// Output stage: the reference's cpu_reference (tools/charsiu_matmul.c:64-77)
//   v = (float)acc * mult + (float)zp_out;  rq = floor(v + 0.5)
// and the NPU's form (src/job.c:137-177) out = clamp(max(rq + L, 0) + O,
// -128, 127) with the lift L = 128 taken in the requant domain and the offset
// O = -128 (zp_out already inside rq). For rq >= -128 the floor never binds
// and out = clamp(rq); below it both forms give -128. So the two are the same
// function, computed here with the reference's roundings.
__device__ __forceinline__ int8_t output_stage(int64_t acc, float mult, float zp_out)
{
	const float v = __fadd_rn(__fmul_rn(__ll2float_rn(acc), mult), zp_out);
	const float rq = floorf(__fadd_rn(v, 0.5f));
	float o = fmaxf(__fadd_rn(rq, 128.0f), 0.0f);     // the fused floor, after the lift
	o = __fadd_rn(o, -128.0f);                        // the offset takes the lift back
	o = fminf(fmaxf(o, -128.0f), 127.0f);
	return (int8_t)__float2int_rz(o);
}

struct I8Params {
	const uint8_t *a, *w;
	const int32_t *bias;
	int8_t *out;
	uint32_t m, k, n;
	float mult, zp_out;
	int zp_a, zp_w;
	// a direct host call (out is mapped host memory): the last CTA to finish
	// raises *done_flag = seq once every byte is visible to the host; null: none
	uint32_t *done_count;      // device, zero between launches
	uint32_t *done_flag;
	uint32_t seq;
};

// The end of a direct call: this CTA's stores reach thread 0 through the
// barrier and are released at device scope by its count; the last CTA
// acquires them all and orders them before the flag with one system fence.
// Every thread of the CTA calls it.
__device__ __forceinline__ void i8_raise_flag(uint32_t *done_count, uint32_t *done_flag,
					      uint32_t seq)
{
	__syncthreads();
	if (threadIdx.x == 0 &&
	    atom_add_acq_rel_gpu(done_count, 1u) == gridDim.x * gridDim.y - 1) {
		*done_count = 0;
		__threadfence_system();
		*(volatile uint32_t *)done_flag = seq;
	}
}

// CUDA cores, dp4a: a 32 (m) x 32 (n) tile per 256-thread CTA, K in steps of
// 64 through shared memory; each thread keeps 4 m rows of one column.
constexpr int I8_TK = 64;
constexpr int I8_PAD = I8_TK + 4;

// The operands of a small job carried in the launch's own parameters (a
// direct host call): a [m][k] at byte 0, w [n][k] at off_w, bias [n] at off_b;
// out is mapped host memory, and the last CTA to finish raises *done_flag =
// seq once every byte of it is visible to the host.
// The launch copies the whole parameter block, so the block comes in three
// sizes (words of 16 bytes) and a job takes the smallest that holds it.
constexpr uint32_t I8_INLINE_BYTES = 30 * 1024;

template <int W>
struct I8Inline {
	I8Params p;
	uint32_t off_w, off_b;
	uint32_t *done_count;      // device, zero between launches
	uint32_t *done_flag;       // mapped host memory
	uint32_t seq;
	uint4 data[W];
};
constexpr int I8_INLINE_W0 = 384, I8_INLINE_W1 = 1280, I8_INLINE_W2 = I8_INLINE_BYTES / 16;
static_assert(sizeof(I8Inline<I8_INLINE_W2>) <= 32764, "kernel parameter space");

__device__ __forceinline__ void i8mm_simt_body(const I8Params &p, const uint8_t *pa,
					       const uint8_t *pw, const int32_t *pbias)
{
	__shared__ __align__(16) int8_t As[32][I8_PAD];
	__shared__ __align__(16) int8_t Ws[32][I8_PAD];
	const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
	const uint32_t m0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
	int acc[4] = {0, 0, 0, 0}, sa[4] = {0, 0, 0, 0}, sw = 0;

	for (uint32_t k0 = 0; k0 < p.k; k0 += I8_TK) {
		for (int i = threadIdx.x; i < 32 * I8_TK; i += 256) {
			const int rr = i / I8_TK, kk = i % I8_TK;
			const uint32_t gk = k0 + kk;
			const uint32_t ma = m0 + rr, nw = n0 + rr;
			As[rr][kk] = (ma < p.m && gk < p.k) ? (int8_t)(pa[(uint64_t)ma * p.k + gk] ^ 0x80) : 0;
			Ws[rr][kk] = (nw < p.n && gk < p.k) ? (int8_t)(pw[(uint64_t)nw * p.k + gk] ^ 0x80) : 0;
		}
		__syncthreads();
#pragma unroll 4
		for (int kk = 0; kk < I8_TK; kk += 4) {
			const uint32_t wv = *reinterpret_cast<const uint32_t *>(&Ws[tx][kk]);
			sw = dp4a_ss(wv, 0x01010101u, sw);
#pragma unroll
			for (int j = 0; j < 4; j++) {
				const uint32_t av = *reinterpret_cast<const uint32_t *>(&As[ty + 8 * j][kk]);
				acc[j] = dp4a_ss(av, wv, acc[j]);
				sa[j] = dp4a_ss(av, 0x01010101u, sa[j]);
			}
		}
		__syncthreads();
	}
	// (no early return: the direct calls' flag needs every thread at a barrier)
	const uint32_t col = n0 + tx;
	if (col < p.n) {
		const int64_t ca = 128 - p.zp_a, cw = 128 - p.zp_w;
#pragma unroll
		for (int j = 0; j < 4; j++) {
			const uint32_t row = m0 + ty + 8 * j;
			if (row >= p.m)
				continue;
			const int64_t total = (int64_t)pbias[col] + acc[j] + cw * sa[j] + ca * sw +
					      (int64_t)p.k * ca * cw;
			p.out[(uint64_t)row * p.n + col] = output_stage(total, p.mult, p.zp_out);
		}
	}
}

// M = 1 (a matvec): a warp per output column, 16 columns a CTA of 8 warps.
// A lane reads 16-byte chunks lane, lane + 32, ... of the column's weight
// row (bytes one by one when K is not a multiple of 16, the rows then not
// being aligned) and the same chunks of the activation; the three integer
// sums of i8mm_simt_body (exact in any order) meet in a warp reduction, and
// the column's output stage is the same. The CTA's 16 output bytes leave in
// one 16-byte store when they are all there and aligned (out may be mapped
// host memory). Against the tiled form (i8mm_simt_body, 32x32 tiles) at
// (1,512,1024): 64 CTAs instead of 32, and 16-byte loads instead of a K loop
// of byte loads through shared memory.
constexpr uint32_t I8MV_COLS = 16;

__global__ void __launch_bounds__(256) i8mv_kernel(const __grid_constant__ I8Params p)
{
	__shared__ __align__(16) int8_t ob[I8MV_COLS];
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const uint32_t c0 = blockIdx.x * I8MV_COLS;
	const bool vec = (p.k & 15u) == 0;
	const int64_t ca = 128 - p.zp_a, cw = 128 - p.zp_w;
#pragma unroll
	for (int h = 0; h < 2; h++) {
		const uint32_t col = c0 + warp + 8 * h;
		int acc = 0, sw = 0, sa = 0;
		if (col < p.n) {
			const uint8_t *wr = p.w + (uint64_t)col * p.k;
			if (vec) {
				for (uint32_t c = lane; c < p.k / 16; c += 32) {
					const uint4 wv = ldg_stream(wr + (size_t)c * 16);
					const uint4 av = *reinterpret_cast<const uint4 *>(p.a + (size_t)c * 16);
					const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
					const uint32_t aa[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
					for (int j = 0; j < 4; j++) {
						const uint32_t ws = ww[j] ^ 0x80808080u, as = aa[j] ^ 0x80808080u;
						acc = dp4a_ss(as, ws, acc);
						sw = dp4a_ss(ws, 0x01010101u, sw);
						sa = dp4a_ss(as, 0x01010101u, sa);
					}
				}
			} else {
				for (uint32_t kk = lane; kk < p.k; kk += 32) {
					const int av = (int)p.a[kk] - 128, wv = (int)wr[kk] - 128;
					acc += av * wv;
					sw += wv;
					sa += av;
				}
			}
		}
		acc = __reduce_add_sync(0xffffffffu, acc);
		sw = __reduce_add_sync(0xffffffffu, sw);
		sa = __reduce_add_sync(0xffffffffu, sa);
		if (lane == 0 && col < p.n) {
			const int64_t total = (int64_t)p.bias[col] + acc + cw * sa + ca * sw +
					      (int64_t)p.k * ca * cw;
			ob[warp + 8 * h] = output_stage(total, p.mult, p.zp_out);
		}
	}
	__syncthreads();
	if (threadIdx.x == 0) {
		const uint32_t cnt = p.n - c0 < I8MV_COLS ? p.n - c0 : I8MV_COLS;
		if (cnt == I8MV_COLS && (c0 & 15u) == 0)
			*reinterpret_cast<uint4 *>(p.out + c0) = *reinterpret_cast<const uint4 *>(ob);
		else
			for (uint32_t j = 0; j < cnt; j++)
				p.out[c0 + j] = ob[j];
	}
	if (p.done_flag)
		i8_raise_flag(p.done_count, p.done_flag, p.seq);
}

template <int W>
__global__ void __launch_bounds__(256)
i8mm_simt_inline_kernel(const __grid_constant__ I8Inline<W> a)
{
	const uint8_t *base = reinterpret_cast<const uint8_t *>(a.data);
	i8mm_simt_body(a.p, base, base + a.off_w, reinterpret_cast<const int32_t *>(base + a.off_b));
	i8_raise_flag(a.done_count, a.done_flag, a.seq);
}

} // namespace cgpu
