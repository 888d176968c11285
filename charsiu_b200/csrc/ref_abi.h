// SPDX-License-Identifier: GPL-2.0-or-later
// The byte layouts of the charsiu structs this layer reads, so it can
// take them by pointer without including charsiu's headers. They must match
// the reference's definitions field for field on LP64 (x86-64, aarch64):
//   struct gguf_tensor    include/charsiu_llm.h:51-59
//   struct charsiu_act    include/charsiu_llm.h:100-119
//   struct charsiu_matmul include/charsiu.h:113-119
//   struct charsiu_job    include/charsiu.h:194-225
//   struct npu_tensor     include/charsiu_llm.h:143-161
// tests/test_abi.py compiles these against the reference headers and
// compares every offset.
#pragma once

#include <cstddef>
#include <cstdint>

namespace cgpu {

struct RefGgufTensor {
	char name[80];
	unsigned n_dims;
	uint64_t ne[4];
	uint32_t type;
	uint64_t offset;
	const void *data;
	uint64_t nbytes;
};

struct RefAct {
	const float *f;
	int n;
	int nb;
	int8_t *q;
	float *d;
	float *bs;
	int quantised;
	int8_t *q1;
	float d1;
	int q1_valid;
};

struct RefMatmul {
	unsigned m, k, n;
	int wdtype, adtype;      // enum charsiu_dtype: INT8 0, INT4 1, FP16 2
};

struct RefJob {
	RefMatmul mm;
	uint32_t input_addr, weight_addr, output_addr, coef_addr;
	float input_scale, weight_scale, output_scale;
	int input_zero_point, weight_zero_point, output_zero_point;
	int acc_out;
};

struct RefNpuTensor {
	int8_t *q;               // [n][k]
	float *scale;            // n * ngroup
	uint64_t kgroup;         // 0 or k: one scale a row
	float *kscale;           // NULL when off
	double *astat;
	uint64_t acalls;
	double *acov;
	float *xcal;
	unsigned nxcal;
	int32_t *wsum;
	uint64_t n, k;
	double rms_rel;
	float out_scale;
	double out_clip;
	uint64_t out_calls;
	float amax_lo, amax_hi;
	char name[80];
};

static_assert(sizeof(RefGgufTensor) == 152, "gguf_tensor layout");
static_assert(sizeof(RefNpuTensor) == 216, "npu_tensor layout");
static_assert(offsetof(RefNpuTensor, kgroup) == 16 && offsetof(RefNpuTensor, kscale) == 24,
	      "npu_tensor.kgroup/kscale");
static_assert(offsetof(RefNpuTensor, n) == 80 && offsetof(RefNpuTensor, k) == 88,
	      "npu_tensor.n/k");
static_assert(offsetof(RefNpuTensor, name) == 136, "npu_tensor.name");
static_assert(offsetof(RefAct, q1) == 48 && offsetof(RefAct, d1) == 56, "charsiu_act.q1/d1");
static_assert(offsetof(RefGgufTensor, ne) == 88, "gguf_tensor.ne");
static_assert(offsetof(RefGgufTensor, type) == 120, "gguf_tensor.type");
static_assert(offsetof(RefGgufTensor, data) == 136, "gguf_tensor.data");
static_assert(sizeof(RefAct) == 64, "charsiu_act layout");
static_assert(offsetof(RefAct, q) == 16 && offsetof(RefAct, d) == 24, "charsiu_act.q/d");
static_assert(offsetof(RefAct, quantised) == 40, "charsiu_act.quantised");
static_assert(sizeof(RefJob) == 64, "charsiu_job layout");
static_assert(offsetof(RefJob, input_scale) == 36, "charsiu_job.input_scale");

constexpr int REF_INT8 = 0;

} // namespace cgpu
