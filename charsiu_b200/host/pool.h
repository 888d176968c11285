// SPDX-License-Identifier: GPL-2.0-or-later
/*
 * A small fork-join pool for the decode's CPU steps (attention heads, the
 * SiLU gate). Each job is `items` independent calls fn(arg, i); which thread
 * runs which item does not change any result, because the items share no
 * accumulator. Workers spin briefly between jobs (the decode issues one
 * every few tens of microseconds), then sleep on a condition variable.
 */
#ifndef CHARSIU_POOL_H
#define CHARSIU_POOL_H

struct pool;

/* `threads` workers besides the caller; NULL when threads < 1 or on failure
 * (the caller then runs every item itself: pool_run accepts NULL). */
struct pool *pool_new(int threads);
void pool_free(struct pool *p);
void pool_run(struct pool *p, void (*fn)(void *arg, int item), void *arg, int items);

#endif
