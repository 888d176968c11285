// SPDX-License-Identifier: GPL-2.0-or-later
/*
 * The GPU layer's struct-form entry points called with charsiu's own structs,
 * as charsiu's code calls them. TEST INFRASTRUCTURE ONLY: oracle/Makefile
 * compiles this file against the reference's headers (include/charsiu.h,
 * include/charsiu_llm.h) into oracle/_ref/libcharsiu_ref_gpu.so, beside the
 * reference's decode loop with the GPU routing applied (route_llama.py), and
 * links it to libcharsiu_gpu.so. The tests compare what these return with the
 * reference's own gguf_matvec and cpu_reference.
 *
 *   refgpu_matvec      charsiu_gpu_add(struct gguf_tensor *) for each of n
 *                      tensors, charsiu_act_set on x (the reference's
 *                      quantiser), then charsiu_gpu_matvec(struct charsiu_act *)
 *                      per tensor or one charsiu_gpu_matvec_group
 *   refgpu_matmul_i8   charsiu_gpu_matmul_i8(struct charsiu_job *) on a job
 *                      filled as tools/charsiu_matmul.c fills one
 */
#define _POSIX_C_SOURCE 200809L

#include <stdio.h>
#include <string.h>

#include "charsiu.h"
#include "charsiu_llm.h"
#include "charsiu_gpu.h"

/*
 * n (1..8) tensors of one type and K, tensor i's N x K/32 GGML blocks at
 * blocks[i], all of N rows; y is [n][N]. group: one charsiu_gpu_matvec_group
 * call instead of n charsiu_gpu_matvec calls. Returns 0, or a negative step
 * number on failure. Adding a tensor twice must give the same id (the
 * routing's lazy registration depends on it): checked too.
 */
int refgpu_matvec(uint32_t type, const void *const *blocks, unsigned n, uint64_t k,
		  uint64_t rows, const float *x, float *y, int group)
{
	struct gguf_tensor w[8];
	struct charsiu_act a;
	struct charsiu_gpu *g;
	float *ys[8];
	int ids[8];
	int rc = 0;

	if (n < 1 || n > 8)
		return -1;
	if (charsiu_act_alloc(&a, (int)k) < 0)
		return -2;
	charsiu_act_set(&a, x, (int)k);
	g = charsiu_gpu_open((unsigned)k, (unsigned)rows, n);
	if (!g) {
		charsiu_act_free(&a);
		return -3;
	}
	memset(w, 0, sizeof(w));
	for (unsigned i = 0; i < n; i++) {
		snprintf(w[i].name, sizeof(w[i].name), "probe.%u.weight", i);
		w[i].n_dims = 2;
		w[i].ne[0] = k;
		w[i].ne[1] = rows;
		w[i].ne[2] = w[i].ne[3] = 1;
		w[i].type = type;
		w[i].data = blocks[i];
		ids[i] = charsiu_gpu_add(g, &w[i]);
		ys[i] = y + (size_t)i * rows;
		if (ids[i] < 0 || charsiu_gpu_add(g, &w[i]) != ids[i]) {
			rc = -4;
			goto out;
		}
	}
	if (group) {
		if (charsiu_gpu_matvec_group(g, ids, n, &a, ys))
			rc = -5;
	} else {
		for (unsigned i = 0; i < n && !rc; i++)
			if (charsiu_gpu_matvec(g, ids[i], &a, ys[i]))
				rc = -6;
	}
out:
	charsiu_gpu_close(g);
	charsiu_act_free(&a);
	return rc;
}

/* The int8 matmul with the NPU output stage, from a charsiu_job. */
int refgpu_matmul_i8(unsigned m, unsigned k, unsigned n, const uint8_t *a, const uint8_t *w,
		     const int32_t *bias, float in_scale, float wt_scale, float out_scale,
		     int in_zp, int wt_zp, int out_zp, int8_t *out)
{
	struct charsiu_job job;
	struct charsiu_gpu *g;
	int rc;

	memset(&job, 0, sizeof(job));
	job.mm.m = m;
	job.mm.k = k;
	job.mm.n = n;
	job.mm.wdtype = CHARSIU_INT8;
	job.mm.adtype = CHARSIU_INT8;
	job.input_scale = in_scale;
	job.weight_scale = wt_scale;
	job.output_scale = out_scale;
	job.input_zero_point = in_zp;
	job.weight_zero_point = wt_zp;
	job.output_zero_point = out_zp;
	g = charsiu_gpu_open(k < 32 ? 32 : (k + 31) / 32 * 32, n, 1);
	if (!g)
		return -3;
	rc = charsiu_gpu_matmul_i8(g, &job, a, w, bias, out);
	charsiu_gpu_close(g);
	return rc;
}
