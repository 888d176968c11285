// SPDX-License-Identifier: GPL-2.0-or-later
// Inline-PTX helpers for the sm_100a tensor cores (tcgen05): tensor-memory
// allocation, the kind::i8 MMA (signed int8 x signed int8 -> int32), its
// commit to an mbarrier, loads of the accumulator out of tensor memory, and
// the two 64-bit descriptors. cta_group::1 throughout; every copy has one destination CTA.
#pragma once

#include <cstdint>

#include "ptx.cuh"

namespace cgpu {

// ---- tensor memory ---------------------------------------------------------

// Allocate `ncols` columns (a power of two, >= 32) of this CTA's tensor memory;
// the base address lands in *dst (shared memory). One whole warp executes it.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols)
{
	asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
		     :: "r"(smem_addr(dst)), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tmem_relinquish()
{
	asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
	asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
		     :: "r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before()
{
	asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after()
{
	asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---- descriptors -------------------------------------------------------------

// Shared-memory matrix descriptor, K-major, no swizzle: the operand is made
// of 8-row x 16-byte core matrices (rows 16 bytes apart); `lbo` is the byte
// distance between the two 16-byte K chunks of one K = 32 step, `sbo` the
// distance between consecutive 8-row groups. Version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc_k_nosw(const void *base, uint32_t lbo, uint32_t sbo)
{
	const uint64_t a = smem_addr(base);
	return ((a >> 4) & 0x3fffull) | (((uint64_t)(lbo >> 4) & 0x3fffull) << 16) |
	       (((uint64_t)(sbo >> 4) & 0x3fffull) << 32) | (1ull << 46);
}

// Instruction descriptor of a dense kind::i8 MMA: D int32, A and B signed
// int8, both K-major, M = m rows (64 or 128), N = n columns (multiple of 16
// for M = 128, 16..256).
__host__ __device__ constexpr uint32_t idesc_i8(uint32_t m, uint32_t n)
{
	return (2u << 4)               // D format: s32
	     | (1u << 7)               // A format: signed 8 bit
	     | (1u << 10)              // B format: signed 8 bit
	     | ((n >> 3) << 17)        // N >> 3
	     | ((m >> 4) << 24);       // M >> 4
}

// ---- the MMA -----------------------------------------------------------------

// D[tmem] (+)= A[smem] . B[smem]^T for one K = 32 step. One thread issues it.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
				       uint32_t idesc, bool accumulate)
{
	asm volatile("{\n\t.reg .pred p;\n\t"
		     "setp.ne.b32 p, %4, 0;\n\t"
		     "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
		     :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc),
			"r"((uint32_t)accumulate)
		     : "memory");
}

// Arrive (once) on `bar` when every tcgen05 op this thread issued before has
// completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar)
{
	asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
		     :: "r"(smem_addr(bar)) : "memory");
}

// ---- accumulator out of tensor memory -----------------------------------------

// 32 lanes x 32 bits, 16 consecutive columns: lane i of the warp gets row
// (its warp's lane quarter base + i), columns col..col+15.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16])
{
	asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
		     "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
		     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
		       "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
		       "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
		     : "r"(taddr));
}

// 32 lanes x 32 bits, 8 consecutive columns
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8])
{
	asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 "
		     "{%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
		     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
		       "=r"(r[6]), "=r"(r[7])
		     : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld()
{
	asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Four blocks' tiles of one chunk (block j at taddr + j * stride; 32 lanes x
// 8 columns each) loaded, waited for, and packed in column pairs in one asm
// statement, so the loaded registers feed packed fp32x2 operations directly.
// MAGIC: each int32 t becomes the bits of the float 1.5 * 2^23 + t
// (|t| < 2^22; see small_int_to_float); otherwise the words are kept as they
// are (tensor memory already holds 1.5 * 2^23 + t).
template <bool MAGIC>
__device__ __forceinline__ void tmem_ld_chunk4(uint32_t taddr, uint32_t stride, uint64_t (&p)[4][4])
{
	if (MAGIC)
		asm volatile("{\n\t.reg .b32 r<32>;\n\t"
			     "tcgen05.ld.sync.aligned.32x32b.x8.b32 {r0, r1, r2, r3, r4, r5, r6, r7}, [%16];\n\t"
			     "tcgen05.ld.sync.aligned.32x32b.x8.b32 {r8, r9, r10, r11, r12, r13, r14, r15}, [%17];\n\t"
			     "tcgen05.ld.sync.aligned.32x32b.x8.b32 {r16, r17, r18, r19, r20, r21, r22, r23}, [%18];\n\t"
			     "tcgen05.ld.sync.aligned.32x32b.x8.b32 {r24, r25, r26, r27, r28, r29, r30, r31}, [%19];\n\t"
			     "tcgen05.wait::ld.sync.aligned;\n\t"
			     "add.u32 r0, r0, 0x4b400000;\n\t"
			     "add.u32 r1, r1, 0x4b400000;\n\t"
			     "add.u32 r2, r2, 0x4b400000;\n\t"
			     "add.u32 r3, r3, 0x4b400000;\n\t"
			     "add.u32 r4, r4, 0x4b400000;\n\t"
			     "add.u32 r5, r5, 0x4b400000;\n\t"
			     "add.u32 r6, r6, 0x4b400000;\n\t"
			     "add.u32 r7, r7, 0x4b400000;\n\t"
			     "add.u32 r8, r8, 0x4b400000;\n\t"
			     "add.u32 r9, r9, 0x4b400000;\n\t"
			     "add.u32 r10, r10, 0x4b400000;\n\t"
			     "add.u32 r11, r11, 0x4b400000;\n\t"
			     "add.u32 r12, r12, 0x4b400000;\n\t"
			     "add.u32 r13, r13, 0x4b400000;\n\t"
			     "add.u32 r14, r14, 0x4b400000;\n\t"
			     "add.u32 r15, r15, 0x4b400000;\n\t"
			     "add.u32 r16, r16, 0x4b400000;\n\t"
			     "add.u32 r17, r17, 0x4b400000;\n\t"
			     "add.u32 r18, r18, 0x4b400000;\n\t"
			     "add.u32 r19, r19, 0x4b400000;\n\t"
			     "add.u32 r20, r20, 0x4b400000;\n\t"
			     "add.u32 r21, r21, 0x4b400000;\n\t"
			     "add.u32 r22, r22, 0x4b400000;\n\t"
			     "add.u32 r23, r23, 0x4b400000;\n\t"
			     "add.u32 r24, r24, 0x4b400000;\n\t"
			     "add.u32 r25, r25, 0x4b400000;\n\t"
			     "add.u32 r26, r26, 0x4b400000;\n\t"
			     "add.u32 r27, r27, 0x4b400000;\n\t"
			     "add.u32 r28, r28, 0x4b400000;\n\t"
			     "add.u32 r29, r29, 0x4b400000;\n\t"
			     "add.u32 r30, r30, 0x4b400000;\n\t"
			     "add.u32 r31, r31, 0x4b400000;\n\t"
			     "mov.b64 %0, {r0, r1};\n\t"
			     "mov.b64 %1, {r2, r3};\n\t"
			     "mov.b64 %2, {r4, r5};\n\t"
			     "mov.b64 %3, {r6, r7};\n\t"
			     "mov.b64 %4, {r8, r9};\n\t"
			     "mov.b64 %5, {r10, r11};\n\t"
			     "mov.b64 %6, {r12, r13};\n\t"
			     "mov.b64 %7, {r14, r15};\n\t"
			     "mov.b64 %8, {r16, r17};\n\t"
			     "mov.b64 %9, {r18, r19};\n\t"
			     "mov.b64 %10, {r20, r21};\n\t"
			     "mov.b64 %11, {r22, r23};\n\t"
			     "mov.b64 %12, {r24, r25};\n\t"
			     "mov.b64 %13, {r26, r27};\n\t"
			     "mov.b64 %14, {r28, r29};\n\t"
			     "mov.b64 %15, {r30, r31};\n\t"
			     "}"
			     : "=l"(p[0][0]), "=l"(p[0][1]), "=l"(p[0][2]), "=l"(p[0][3]), "=l"(p[1][0]), "=l"(p[1][1]), "=l"(p[1][2]), "=l"(p[1][3]), "=l"(p[2][0]), "=l"(p[2][1]), "=l"(p[2][2]), "=l"(p[2][3]), "=l"(p[3][0]), "=l"(p[3][1]), "=l"(p[3][2]), "=l"(p[3][3])
			     : "r"(taddr), "r"(taddr + stride), "r"(taddr + 2 * stride), "r"(taddr + 3 * stride)
			     : "memory");
	else
		asm volatile("{\n\t.reg .b32 r<32>;\n\t"
			     "tcgen05.ld.sync.aligned.32x32b.x8.b32 {r0, r1, r2, r3, r4, r5, r6, r7}, [%16];\n\t"
			     "tcgen05.ld.sync.aligned.32x32b.x8.b32 {r8, r9, r10, r11, r12, r13, r14, r15}, [%17];\n\t"
			     "tcgen05.ld.sync.aligned.32x32b.x8.b32 {r16, r17, r18, r19, r20, r21, r22, r23}, [%18];\n\t"
			     "tcgen05.ld.sync.aligned.32x32b.x8.b32 {r24, r25, r26, r27, r28, r29, r30, r31}, [%19];\n\t"
			     "tcgen05.wait::ld.sync.aligned;\n\t"
			     "mov.b64 %0, {r0, r1};\n\t"
			     "mov.b64 %1, {r2, r3};\n\t"
			     "mov.b64 %2, {r4, r5};\n\t"
			     "mov.b64 %3, {r6, r7};\n\t"
			     "mov.b64 %4, {r8, r9};\n\t"
			     "mov.b64 %5, {r10, r11};\n\t"
			     "mov.b64 %6, {r12, r13};\n\t"
			     "mov.b64 %7, {r14, r15};\n\t"
			     "mov.b64 %8, {r16, r17};\n\t"
			     "mov.b64 %9, {r18, r19};\n\t"
			     "mov.b64 %10, {r20, r21};\n\t"
			     "mov.b64 %11, {r22, r23};\n\t"
			     "mov.b64 %12, {r24, r25};\n\t"
			     "mov.b64 %13, {r26, r27};\n\t"
			     "mov.b64 %14, {r28, r29};\n\t"
			     "mov.b64 %15, {r30, r31};\n\t"
			     "}"
			     : "=l"(p[0][0]), "=l"(p[0][1]), "=l"(p[0][2]), "=l"(p[0][3]), "=l"(p[1][0]), "=l"(p[1][1]), "=l"(p[1][2]), "=l"(p[1][3]), "=l"(p[2][0]), "=l"(p[2][1]), "=l"(p[2][2]), "=l"(p[2][3]), "=l"(p[3][0]), "=l"(p[3][1]), "=l"(p[3][2]), "=l"(p[3][3])
			     : "r"(taddr), "r"(taddr + stride), "r"(taddr + 2 * stride), "r"(taddr + 3 * stride)
			     : "memory");
}

// The same for one block, for a chunk's ragged tail.
template <bool MAGIC>
__device__ __forceinline__ void tmem_ld_block(uint32_t taddr, uint64_t (&p)[4])
{
	if (MAGIC)
		asm volatile("{\n\t.reg .b32 r<8>;\n\t"
			     "tcgen05.ld.sync.aligned.32x32b.x8.b32 {r0, r1, r2, r3, r4, r5, r6, r7}, [%4];\n\t"
			     "tcgen05.wait::ld.sync.aligned;\n\t"
			     "add.u32 r0, r0, 0x4b400000;\n\t"
			     "add.u32 r1, r1, 0x4b400000;\n\t"
			     "add.u32 r2, r2, 0x4b400000;\n\t"
			     "add.u32 r3, r3, 0x4b400000;\n\t"
			     "add.u32 r4, r4, 0x4b400000;\n\t"
			     "add.u32 r5, r5, 0x4b400000;\n\t"
			     "add.u32 r6, r6, 0x4b400000;\n\t"
			     "add.u32 r7, r7, 0x4b400000;\n\t"
			     "mov.b64 %0, {r0, r1};\n\t"
			     "mov.b64 %1, {r2, r3};\n\t"
			     "mov.b64 %2, {r4, r5};\n\t"
			     "mov.b64 %3, {r6, r7};\n\t"
			     "}"
			     : "=l"(p[0]), "=l"(p[1]), "=l"(p[2]), "=l"(p[3])
			     : "r"(taddr)
			     : "memory");
	else
		asm volatile("{\n\t.reg .b32 r<8>;\n\t"
			     "tcgen05.ld.sync.aligned.32x32b.x8.b32 {r0, r1, r2, r3, r4, r5, r6, r7}, [%4];\n\t"
			     "tcgen05.wait::ld.sync.aligned;\n\t"
			     "mov.b64 %0, {r0, r1};\n\t"
			     "mov.b64 %1, {r2, r3};\n\t"
			     "mov.b64 %2, {r4, r5};\n\t"
			     "mov.b64 %3, {r6, r7};\n\t"
			     "}"
			     : "=l"(p[0]), "=l"(p[1]), "=l"(p[2]), "=l"(p[3])
			     : "r"(taddr)
			     : "memory");
}

// Four blocks' tiles of one chunk, 32 lanes x 4 columns each (an epilogue
// warp that owns 4 activations), with the integer-to-float add of
// tmem_ld_chunk4<true>: p[j] = block j's columns in pairs.
__device__ __forceinline__ void tmem_ld_chunk4_c4(uint32_t taddr, uint32_t stride,
						  uint64_t (&p)[4][2])
{
	asm volatile("{\n\t.reg .b32 r<16>;\n\t"
		     "tcgen05.ld.sync.aligned.32x32b.x4.b32 {r0, r1, r2, r3}, [%8];\n\t"
		     "tcgen05.ld.sync.aligned.32x32b.x4.b32 {r4, r5, r6, r7}, [%9];\n\t"
		     "tcgen05.ld.sync.aligned.32x32b.x4.b32 {r8, r9, r10, r11}, [%10];\n\t"
		     "tcgen05.ld.sync.aligned.32x32b.x4.b32 {r12, r13, r14, r15}, [%11];\n\t"
		     "tcgen05.wait::ld.sync.aligned;\n\t"
		     "add.u32 r0, r0, 0x4b400000;\n\t"
		     "add.u32 r1, r1, 0x4b400000;\n\t"
		     "add.u32 r2, r2, 0x4b400000;\n\t"
		     "add.u32 r3, r3, 0x4b400000;\n\t"
		     "add.u32 r4, r4, 0x4b400000;\n\t"
		     "add.u32 r5, r5, 0x4b400000;\n\t"
		     "add.u32 r6, r6, 0x4b400000;\n\t"
		     "add.u32 r7, r7, 0x4b400000;\n\t"
		     "add.u32 r8, r8, 0x4b400000;\n\t"
		     "add.u32 r9, r9, 0x4b400000;\n\t"
		     "add.u32 r10, r10, 0x4b400000;\n\t"
		     "add.u32 r11, r11, 0x4b400000;\n\t"
		     "add.u32 r12, r12, 0x4b400000;\n\t"
		     "add.u32 r13, r13, 0x4b400000;\n\t"
		     "add.u32 r14, r14, 0x4b400000;\n\t"
		     "add.u32 r15, r15, 0x4b400000;\n\t"
		     "mov.b64 %0, {r0, r1};\n\t"
		     "mov.b64 %1, {r2, r3};\n\t"
		     "mov.b64 %2, {r4, r5};\n\t"
		     "mov.b64 %3, {r6, r7};\n\t"
		     "mov.b64 %4, {r8, r9};\n\t"
		     "mov.b64 %5, {r10, r11};\n\t"
		     "mov.b64 %6, {r12, r13};\n\t"
		     "mov.b64 %7, {r14, r15};\n\t"
		     "}"
		     : "=l"(p[0][0]), "=l"(p[0][1]), "=l"(p[1][0]), "=l"(p[1][1]), "=l"(p[2][0]),
		       "=l"(p[2][1]), "=l"(p[3][0]), "=l"(p[3][1])
		     : "r"(taddr), "r"(taddr + stride), "r"(taddr + 2 * stride), "r"(taddr + 3 * stride)
		     : "memory");
}

// The same for one block, for a chunk's ragged tail.
__device__ __forceinline__ void tmem_ld_block_c4(uint32_t taddr, uint64_t (&p)[2])
{
	asm volatile("{\n\t.reg .b32 r<4>;\n\t"
		     "tcgen05.ld.sync.aligned.32x32b.x4.b32 {r0, r1, r2, r3}, [%2];\n\t"
		     "tcgen05.wait::ld.sync.aligned;\n\t"
		     "add.u32 r0, r0, 0x4b400000;\n\t"
		     "add.u32 r1, r1, 0x4b400000;\n\t"
		     "add.u32 r2, r2, 0x4b400000;\n\t"
		     "add.u32 r3, r3, 0x4b400000;\n\t"
		     "mov.b64 %0, {r0, r1};\n\t"
		     "mov.b64 %1, {r2, r3};\n\t"
		     "}"
		     : "=l"(p[0]), "=l"(p[1])
		     : "r"(taddr)
		     : "memory");
}

// The same 32 lanes x 16 columns, every word set to `v`.
__device__ __forceinline__ void tmem_fill16(uint32_t taddr, uint32_t v)
{
	asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
		     "{%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};"
		     :: "r"(taddr), "r"(v) : "memory");
}

__device__ __forceinline__ void tmem_fill8(uint32_t taddr, uint32_t v)
{
	asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], "
		     "{%1, %1, %1, %1, %1, %1, %1, %1};"
		     :: "r"(taddr), "r"(v) : "memory");
}

__device__ __forceinline__ void tmem_wait_st()
{
	asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// |t| < 2^22 to fp32, exactly: 0x4b400000 is 1.5 * 2^23, whose float spacing
// is 1, so the bits 0x4b400000 + t are the float 1.5 * 2^23 + t, and taking
// 1.5 * 2^23 away again is exact. Two full-rate ops instead of a conversion.
constexpr uint32_t INT_FLOAT_MAGIC = 0x4b400000u;
constexpr float INT_FLOAT_BIAS = 12582912.0f;

__device__ __forceinline__ float small_int_to_float(int32_t t)
{
	return __fsub_rn(__int_as_float((int32_t)INT_FLOAT_MAGIC + t), INT_FLOAT_BIAS);
}

} // namespace cgpu
