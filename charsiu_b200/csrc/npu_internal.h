// SPDX-License-Identifier: GPL-2.0-or-later
// What the decode step (decoder.cu) reads of an NPU-format layer
// (npu_layer.cu) beyond include/charsiu_npu.h. Hidden symbols of the library.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

struct charsiu_npu;

namespace cgpu {

int npu_layer_device(const charsiu_npu *g);
bool npu_layer_dead(const charsiu_npu *g);
// K, rows and the padded row length kp of tensor id; false for an unknown id
bool npu_layer_tensor(const charsiu_npu *g, int id, uint64_t *k, uint64_t *n, uint32_t *kp);
// The tensors ids (one K) against the single-scale activation q1 (kp bytes,
// device, zero past K) whose d1 the kernel reads from device memory once the
// kernel before it is done; ys[i] device pointers; queued on st. 0, or -1.
int npu_layer_matvec_dev_d1(charsiu_npu *g, const int *ids, unsigned n, const int8_t *q1,
			    const float *d1, float *const *ys, cudaStream_t st);
unsigned long npu_layer_launches(const charsiu_npu *g);

} // namespace cgpu
