// SPDX-License-Identifier: GPL-2.0-or-later
// The launch parameters shared by the CUDA-core block-quant matvec kernels
// (qmv1.cuh for one activation, qmvm.cuh for 2, 4 or 8): up to eight tensors
// of one K and quant type in one launch, their 8-row groups numbered through
// in order. All of them compute charsiu's gguf_matvec bit for bit (reference
// src/gguf.c:1061-1107, 1149-1171): per output row
//     s = 0; for b in blocks: s += (d_w[b] * d_a[b]) * (float)t_b
// with t_b the exact int32 dot of block b, every multiply and add rounded on
// its own, left to right. Integer dots can be split any way; the float sum
// cannot, so the kernels compute the terms in parallel and add them in block
// order.
#pragma once

#include "layout.h"
#include "ptx.cuh"

namespace cgpu {

constexpr int QMV_MAX_TENSORS = 8;
constexpr int QMV_MAX_M = 8;
constexpr size_t QMV_SMEM_MAX = 227 * 1024;     // dynamic shared memory a CTA may use

struct QmvTensor {
	const uint8_t *data;     // the device layout of layout.h
	float *y;                // y[m * y_stride + row], rows of this GPU
	uint32_t type, rows, groups, group_end;
	uint32_t y_stride;
	uint32_t pad_;
};

struct QmvParams {
	QmvTensor t[QMV_MAX_TENSORS];
	uint32_t ntensor, total_groups, k, nb;
	const int8_t *q;         // activation quants [M][nb * 32]
	const float *d;          // activation deltas [M][nb]
	int *err;                // set nonzero if a wait gave up (mapped host memory)
	// direct host calls (M = 1): when done_flag is set, the last CTA to
	// finish writes `seq` there (mapped host memory) once every y is visible
	// to the host, and the kernel time since *t_start there + 1
	uint32_t *done_count;    // device, zero between launches
	uint32_t *done_flag;     // [0] seq, [1] kernel ns
	unsigned long long *t_start;
	uint32_t seq;
	// 1: let the next launch start as soon as every CTA of this one has
	// started (its weights then stream in while this one computes); 0: once
	// every CTA has staged the activation
	uint32_t early_trigger;
};

} // namespace cgpu
