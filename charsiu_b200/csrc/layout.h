// SPDX-License-Identifier: GPL-2.0-or-later
// The device layout of a q8_0 / q4_0 tensor, fixed at add time.
//
// A GGUF tensor is N rows of K/32 blocks, each block an fp16 delta followed
// by the quants (34 bytes q8_0, 18 bytes q4_0; reference src/gguf.c:446-447).
// Those 34- and 18-byte records cannot be read with aligned 16-byte vectors,
// so at add time they are split and regrouped:
//
//   rows in GROUPS of RG = 8; a group's K in SEGMENTS of SB = 16 blocks;
//   a segment of sb blocks (sb = SB, or fewer for the last) is one contiguous
//   run of bytes:
//       quants  [sb][QB / 16 chunks][RG rows][16 B]   QB = 32 (q8_0), 16 (q4_0)
//       deltas  [sb][RG rows]                          fp16, unchanged bits
//   a group is its segments back to back, a tensor its groups back to back.
//
// So one segment is one bulk copy, 8 lanes reading 16 bytes each of one chunk
// cover 128 contiguous bytes, and each (group, block, chunk) is an 8-row x
// 16-byte core matrix of the tensor cores' K-major no-swizzle operand layout:
// a 128-row MMA tile of one block is 16 groups' core-matrix pairs, K-chunk
// stride 128 B, 8-row stride one segment. Rows past N in the last group are
// zero (delta 0, quants 0) and are never written out. q4_0 nibbles keep GGUF
// order (byte j: low nibble element j, high nibble element j + 16).
#pragma once

#include <cstdint>

namespace cgpu {

constexpr int RG = 8;        // rows per group
constexpr int SB = 16;       // blocks per segment
constexpr uint32_t TYPE_Q4_0 = 2;
constexpr uint32_t TYPE_Q8_0 = 8;

__host__ __device__ constexpr uint32_t quant_bytes(uint32_t type)
{
	return type == TYPE_Q8_0 ? 32u : 16u;
}

// bytes one block of one group occupies (RG rows of quants + RG deltas)
__host__ __device__ constexpr uint32_t block_group_bytes(uint32_t type)
{
	return RG * (quant_bytes(type) + 2u);
}

__host__ __device__ inline uint64_t group_bytes(uint32_t type, uint32_t nb)
{
	return (uint64_t)nb * block_group_bytes(type);
}

__host__ __device__ inline uint32_t nsegments(uint32_t nb)
{
	return (nb + SB - 1) / SB;
}

__host__ __device__ inline uint32_t seg_blocks(uint32_t nb, uint32_t seg)
{
	uint32_t left = nb - seg * SB;
	return left < (uint32_t)SB ? left : (uint32_t)SB;
}

// byte offset of segment `seg` within its group
__host__ __device__ inline uint64_t seg_offset(uint32_t type, uint32_t seg)
{
	return (uint64_t)seg * SB * block_group_bytes(type);
}

constexpr uint32_t MAX_SEG_BYTES = SB * RG * (32u + 2u);   // 4352

// byte offset, within its segment, of 16-byte chunk c of row r of block bi
__host__ __device__ constexpr uint32_t quant_offset(uint32_t type, uint32_t bi, uint32_t c,
						    uint32_t r)
{
	return bi * RG * quant_bytes(type) + c * RG * 16 + r * 16;
}

// q6_K (256-weight super-blocks of 210 bytes) has a layout of its own: a row
// is its super-blocks' first 208 bytes (ql[128], qh[64], int8 scales[16]) back
// to back, then their fp16 d's, padded to 16 bytes; rows back to back.
constexpr uint32_t TYPE_Q6_K = 14;

__host__ __device__ inline uint64_t q6k_row_bytes(uint32_t nsb)
{
	return (uint64_t)nsb * 208 + ((nsb * 2u + 15u) & ~15u);
}

} // namespace cgpu
