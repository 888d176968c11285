// SPDX-License-Identifier: GPL-2.0-or-later
/*
 * The reference's own CPU denominators for the int8 matmul, exported. TEST
 * INFRASTRUCTURE ONLY (the CPU baseline of bench.py), compiled by
 * oracle/Makefile into oracle/_ref/libcharsiu_ref.so from the reference's
 * tools/charsiu_bench.c where it lies: that file's cpu_us (:74-95) is
 * `static`, so the file is included here with its main() renamed, as
 * ref_shim.c does for tools/charsiu_matmul.c.
 */
#define _POSIX_C_SOURCE 200809L

#define main charsiu_bench_tool_main
#include "charsiu_bench.c"
#undef main

/* cpu_us: microseconds a call of the one-core int32 MAC loop over the job's
 * shape (activation row a[k], weights w[n][k]), the mean of `reps` calls */
double ref_cpu_us(unsigned m, unsigned k, unsigned n, const uint8_t *a, const uint8_t *w,
		  int in_zp, int wt_zp, unsigned reps)
{
	struct charsiu_job job;

	memset(&job, 0, sizeof(job));
	job.mm.m = m;
	job.mm.k = k;
	job.mm.n = n;
	job.mm.wdtype = CHARSIU_INT8;
	job.mm.adtype = CHARSIU_INT8;
	job.input_zero_point = in_zp;
	job.weight_zero_point = wt_zp;
	return cpu_us(&job, a, w, reps ? reps : 1);
}
