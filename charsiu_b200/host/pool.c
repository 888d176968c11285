// SPDX-License-Identifier: GPL-2.0-or-later
/*
 * The decode's fork-join pool (pool.h). A job is published by bumping `gen`;
 * workers and the caller then take items from the shared counter `next` until
 * it passes `items`, and each worker counts itself in `done`. A worker that
 * has seen no job for SPIN_NS goes to sleep on `cv`; the publisher signals
 * only when someone sleeps (the seq_cst order of `gen` and `sleeping` makes
 * that safe: a worker re-reads `gen` after counting itself asleep).
 */
#define _POSIX_C_SOURCE 200809L

#include "pool.h"

#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <time.h>

#if defined(__x86_64__) || defined(__i386__)
#include <immintrin.h>
#define CPU_RELAX() _mm_pause()
#else
#define CPU_RELAX() ((void)0)
#endif

#define MAX_WORKERS 64
#define SPIN_NS 2000000L            /* 2 ms of spinning before sleeping */

struct pool {
	pthread_t th[MAX_WORKERS];
	int n;
	_Atomic unsigned gen;
	_Atomic int next, done, stop, sleeping;
	void (*fn)(void *, int);
	void *arg;
	int items;
	pthread_mutex_t mu;
	pthread_cond_t cv;
};

static long now_ns(void)
{
	struct timespec t;

	clock_gettime(CLOCK_MONOTONIC, &t);
	return t.tv_sec * 1000000000L + t.tv_nsec;
}

static void take_items(struct pool *p)
{
	int i;

	while ((i = atomic_fetch_add_explicit(&p->next, 1, memory_order_relaxed)) < p->items)
		p->fn(p->arg, i);
}

static void *worker(void *arg)
{
	struct pool *p = arg;
	unsigned seen = 0;

	for (;;) {
		unsigned g;
		long t0 = now_ns();
		int spins = 0;

		while ((g = atomic_load(&p->gen)) == seen) {
			if (atomic_load_explicit(&p->stop, memory_order_relaxed))
				return NULL;
			CPU_RELAX();
			if (++spins & 255)
				continue;
			if (now_ns() - t0 < SPIN_NS)
				continue;
			pthread_mutex_lock(&p->mu);
			atomic_fetch_add(&p->sleeping, 1);
			while (atomic_load(&p->gen) == seen && !atomic_load(&p->stop))
				pthread_cond_wait(&p->cv, &p->mu);
			atomic_fetch_sub(&p->sleeping, 1);
			pthread_mutex_unlock(&p->mu);
			t0 = now_ns();
		}
		if (atomic_load(&p->stop))
			return NULL;
		seen = g;
		take_items(p);
		atomic_fetch_add_explicit(&p->done, 1, memory_order_release);
	}
}

struct pool *pool_new(int threads)
{
	struct pool *p;

	if (threads < 1)
		return NULL;
	if (threads > MAX_WORKERS)
		threads = MAX_WORKERS;
	p = calloc(1, sizeof(*p));
	if (!p)
		return NULL;
	pthread_mutex_init(&p->mu, NULL);
	pthread_cond_init(&p->cv, NULL);
	for (int i = 0; i < threads; i++) {
		if (pthread_create(&p->th[i], NULL, worker, p)) {
			pool_free(p);
			return NULL;
		}
		p->n++;
	}
	return p;
}

void pool_free(struct pool *p)
{
	if (!p)
		return;
	pthread_mutex_lock(&p->mu);
	atomic_store(&p->stop, 1);
	pthread_cond_broadcast(&p->cv);
	pthread_mutex_unlock(&p->mu);
	for (int i = 0; i < p->n; i++)
		pthread_join(p->th[i], NULL);
	pthread_cond_destroy(&p->cv);
	pthread_mutex_destroy(&p->mu);
	free(p);
}

void pool_run(struct pool *p, void (*fn)(void *, int), void *arg, int items)
{
	if (!p || items < 2) {
		for (int i = 0; i < items; i++)
			fn(arg, i);
		return;
	}
	p->fn = fn;
	p->arg = arg;
	p->items = items;
	atomic_store_explicit(&p->next, 0, memory_order_relaxed);
	atomic_store_explicit(&p->done, 0, memory_order_relaxed);
	atomic_fetch_add(&p->gen, 1);          /* publishes fn, arg, items */
	if (atomic_load(&p->sleeping)) {
		pthread_mutex_lock(&p->mu);
		pthread_cond_broadcast(&p->cv);
		pthread_mutex_unlock(&p->mu);
	}
	take_items(p);
	while (atomic_load_explicit(&p->done, memory_order_acquire) < p->n)
		CPU_RELAX();
}
