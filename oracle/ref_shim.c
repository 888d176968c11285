// SPDX-License-Identifier: GPL-2.0-or-later
/*
 * A thin shim over the reference itself, compiled by oracle/Makefile from
 * the reference's own sources where they lie (nothing of them is copied into
 * this repository). The result, oracle/_ref/libcharsiu_ref.so, is TEST
 * INFRASTRUCTURE: it pins the restatement in charsiu_oracle.c and serves as
 * the CPU baseline. It is never part of the product.
 *
 * It adds two things the reference does not export:
 *  - cpu_reference() of tools/charsiu_matmul.c:41-81 is `static`, so that
 *    file is included here with its main() renamed, and a wrapper exports it;
 *  - a charsiu_run-style greedy driver (tools/charsiu_run.c:220-317) that
 *    takes token ids instead of text, because the workload's prompt is a list
 *    of seeded ids.
 */
#define _POSIX_C_SOURCE 200809L

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <time.h>

#include "charsiu.h"
#include "charsiu_llm.h"

/* (REF_SHIM_NO_TOOL: the decode-only builds, whose libraries carry no NPU job
 * code for the tool to call) */
#ifndef REF_SHIM_NO_TOOL
#define main charsiu_matmul_tool_main
#include "charsiu_matmul.c"
#undef main

int ref_cpu_reference(const struct charsiu_job *job, const uint8_t *a,
		      const uint8_t *b, const int32_t *bias, uint8_t *out)
{
	return cpu_reference(job, a, b, bias, out);
}

/* flat arguments, so a ctypes caller needs no struct layout */
int ref_matmul_i8(unsigned m, unsigned k, unsigned n, const uint8_t *a,
		  const uint8_t *w, const int32_t *bias, float in_scale,
		  float wt_scale, float out_scale, int in_zp, int wt_zp,
		  int out_zp, uint8_t *out)
{
	struct charsiu_job job;

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
	return cpu_reference(&job, a, w, bias, out);
}
#endif /* REF_SHIM_NO_TOOL */

size_t ref_sizeof_act(void)
{
	return sizeof(struct charsiu_act);
}

/* charsiu_act_set + gguf_matvec over all rows, on a caller's raw blocks */
int ref_matvec(uint32_t type, const void *blocks, uint64_t k, uint64_t n,
	       const float *x, float *y, int8_t *q_out, float *d_out)
{
	struct gguf_tensor w;
	struct charsiu_act a;

	memset(&w, 0, sizeof(w));
	w.n_dims = 2;
	w.ne[0] = k;
	w.ne[1] = n;
	w.ne[2] = w.ne[3] = 1;
	w.type = type;
	w.data = blocks;
	if (charsiu_act_alloc(&a, (int)k) < 0)
		return -1;
	charsiu_act_set(&a, x, (int)k);
	gguf_matvec(&w, &a, y, 0, n);
	if (q_out)
		memcpy(q_out, a.q, (size_t)a.nb * 32);
	if (d_out)
		memcpy(d_out, a.d, (size_t)a.nb * sizeof(float));
	charsiu_act_free(&a);
	return 0;
}

static double now_ms(void)
{
	struct timespec t;

	clock_gettime(CLOCK_MONOTONIC, &t);
	return (double)t.tv_sec * 1e3 + (double)t.tv_nsec / 1e6;
}

/*
 * The CPU baseline of one matvec: charsiu_act_set of x, then gguf_matvec over
 * all n rows, `reps` times; *ms gets the mean time a call. With threads > 1
 * the rows are split as the decode loop's pool splits them (src/llama.c:63-73:
 * worker i takes rows [i * per, i * per + per) with per = ceil(n / threads))
 * over that many threads, started once and released each call by a barrier,
 * the caller quantising first as matvec() does (src/llama.c:178-182).
 */
struct mv_job {
	const struct gguf_tensor *w;
	const struct charsiu_act *a;
	float *y;
	uint64_t n;
	int threads, reps;
	pthread_barrier_t go, done;
};

struct mv_worker {
	struct mv_job *j;
	int id;
};

static void mv_slice(const struct mv_job *j, int id)
{
	uint64_t per = (j->n + (uint64_t)j->threads - 1) / (uint64_t)j->threads;
	uint64_t r0 = per * (uint64_t)id, cnt;

	if (r0 >= j->n)
		return;
	cnt = j->n - r0 < per ? j->n - r0 : per;
	gguf_matvec(j->w, j->a, j->y, r0, cnt);
}

static void *mv_worker_main(void *arg)
{
	struct mv_worker *wk = arg;

	for (int r = 0; r < wk->j->reps; r++) {
		pthread_barrier_wait(&wk->j->go);
		mv_slice(wk->j, wk->id);
		pthread_barrier_wait(&wk->j->done);
	}
	return NULL;
}

int ref_matvec_time(uint32_t type, const void *blocks, uint64_t k, uint64_t n, const float *x,
		    int threads, int reps, double *ms)
{
	struct gguf_tensor w;
	struct charsiu_act a;
	struct mv_job j;
	pthread_t th[256];
	struct mv_worker wk[256];
	double t0;
	int nt = 0, rc = 0;

	if (threads < 1 || threads > 256 || reps < 1)
		return -1;
	memset(&w, 0, sizeof(w));
	w.n_dims = 2;
	w.ne[0] = k;
	w.ne[1] = n;
	w.ne[2] = w.ne[3] = 1;
	w.type = type;
	w.data = blocks;
	if (charsiu_act_alloc(&a, (int)k) < 0)
		return -1;
	memset(&j, 0, sizeof(j));
	j.w = &w;
	j.a = &a;
	j.y = malloc((size_t)n * sizeof(float));
	j.n = n;
	j.threads = threads;
	j.reps = reps;
	if (!j.y) {
		charsiu_act_free(&a);
		return -1;
	}
	if (threads > 1) {
		pthread_barrier_init(&j.go, NULL, (unsigned)threads);
		pthread_barrier_init(&j.done, NULL, (unsigned)threads);
		for (nt = 0; nt < threads - 1; nt++) {
			wk[nt].j = &j;
			wk[nt].id = nt + 1;
			if (pthread_create(&th[nt], NULL, mv_worker_main, &wk[nt])) {
				rc = -1;
				break;
			}
		}
	}
	if (!rc) {
		t0 = now_ms();
		for (int r = 0; r < reps; r++) {
			charsiu_act_set(&a, x, (int)k);
			if (threads > 1)
				pthread_barrier_wait(&j.go);
			mv_slice(&j, 0);
			if (threads > 1)
				pthread_barrier_wait(&j.done);
		}
		*ms = (now_ms() - t0) / reps;
	}
	for (int i = 0; i < nt; i++)
		pthread_join(th[i], NULL);
	if (threads > 1) {
		pthread_barrier_destroy(&j.go);
		pthread_barrier_destroy(&j.done);
	}
	free(j.y);
	charsiu_act_free(&a);
	return rc;
}

/*
 * Greedy decode through the reference's own llama_load / llama_forward /
 * llama_argmax. Returns the number of tokens written to out, or -1.
 * *gen_ms is the generation time (tools/charsiu_run.c:295-339), and, when
 * logits_out is given, the logits after the prompt are copied into it.
 */
int ref_greedy_timed(const char *path, const int32_t *prompt, int n_prompt,
		     int n_gen, int n_ctx, int32_t *out, double *prompt_ms,
		     double *gen_ms, float *logits_out, double *tok_ms);

int ref_greedy(const char *path, const int32_t *prompt, int n_prompt,
	       int n_gen, int n_ctx, int32_t *out, double *prompt_ms,
	       double *gen_ms, float *logits_out)
{
	return ref_greedy_timed(path, prompt, n_prompt, n_gen, n_ctx, out,
				prompt_ms, gen_ms, logits_out, NULL);
}

/* The same, also stamping tok_ms[i]: ms since the generation loop began when
 * token i's forward pass had finished. */
int ref_greedy_timed(const char *path, const int32_t *prompt, int n_prompt,
		     int n_gen, int n_ctx, int32_t *out, double *prompt_ms,
		     double *gen_ms, float *logits_out, double *tok_ms)
{
	struct llama_model m;
	struct llama_state *st;
	const float *logits = NULL;
	double t0;
	int i;

	if (llama_load(&m, path) < 0)
		return -1;
	st = llama_state_new(&m, n_ctx);
	if (!st) {
		llama_free(&m);
		return -1;
	}
	t0 = now_ms();
	for (i = 0; i < n_prompt; i++)
		logits = llama_forward(st, prompt[i], i);
	if (prompt_ms)
		*prompt_ms = now_ms() - t0;
	if (logits_out && logits)
		memcpy(logits_out, logits, (size_t)m.n_vocab * sizeof(float));
	t0 = now_ms();
	for (i = 0; i < n_gen && logits; i++) {
		out[i] = llama_argmax(logits, m.n_vocab);
		if (st->pos >= st->n_ctx)
			break;
		logits = llama_forward(st, out[i], st->pos);
		if (tok_ms)
			tok_ms[i] = now_ms() - t0;
	}
	if (gen_ms)
		*gen_ms = now_ms() - t0;
	llama_state_free(st);
	llama_free(&m);
	return i;
}

/* ---- the NPU number format (CHARSIU_NPU_QUANT), for the restatement's pins */

/* npu_tensor_build (src/npuquant.c:34-296) on a caller's raw GGUF rows */
int ref_npu_tensor_build(uint32_t type, const void *data, uint64_t k, uint64_t n,
			 int8_t *q, float *scale, int32_t *wsum)
{
	struct gguf_tensor w;
	struct npu_tensor t;

	memset(&w, 0, sizeof(w));
	snprintf(w.name, sizeof(w.name), "probe");
	w.n_dims = 2;
	w.ne[0] = k;
	w.ne[1] = n;
	w.ne[2] = w.ne[3] = 1;
	w.type = type;
	w.data = data;
	if (npu_tensor_build(&t, &w) < 0)
		return -1;
	memcpy(q, t.q, (size_t)n * k);
	memcpy(scale, t.scale, (size_t)n * sizeof(float));
	memcpy(wsum, t.wsum, (size_t)n * sizeof(int32_t));
	npu_tensor_free(&t);
	return 0;
}

/* charsiu_act_set's single-scale activation (src/gguf.c:883-910); valid only
 * in a process whose CHARSIU_NPU_QUANT was set before its first call */
int ref_act_q1(const float *x, int n, int8_t *q1, float *d1)
{
	struct charsiu_act a;
	int rc = -1;

	if (charsiu_act_alloc(&a, n) < 0)
		return -1;
	charsiu_act_set(&a, x, n);
	if (a.q1_valid) {
		memcpy(q1, a.q1, (size_t)a.nb * 32);
		*d1 = a.d1;
		rc = 0;
	}
	charsiu_act_free(&a);
	return rc;
}

/* npu_matvec (src/npuquant.c:447-544), the CPU model, one scale a row */
void ref_npu_matvec(const int8_t *q, const float *scale, uint64_t k, uint64_t n,
		    const int8_t *q1, float d1, float *y)
{
	struct npu_tensor t;
	struct charsiu_act a;

	memset(&t, 0, sizeof(t));
	memset(&a, 0, sizeof(a));
	t.q = (int8_t *)q;
	t.scale = (float *)scale;
	t.kgroup = k;
	t.n = n;
	t.k = k;
	a.n = (int)k;
	a.q1 = (int8_t *)q1;
	a.d1 = d1;
	a.q1_valid = 1;
	npu_matvec(&t, &a, y, 0, n);
}
