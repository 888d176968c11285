// SPDX-License-Identifier: GPL-2.0-or-later
// Host copies of up to 8 segments, as one run of bytes cut into 16 KB items
// for a pool of host threads (host/pool.c) once the run reaches 64 KB: the
// large int8 jobs' operands into the pinned staging buffer and their output
// out of it, and the direct calls' outputs out of mapped host memory. The
// GPU's PCIe writes leave those lines in no CPU cache, so one thread reads
// 64 KB of them in about 8 us; a single thread copies 512 KB of caller memory
// at about 10 GB/s. Which thread copies which item changes no byte.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>

extern "C" {
#include "../host/pool.h"
}

namespace cgpu {

struct ParCopy {
	static constexpr int MAX_SEG = 8;
	static constexpr size_t CHUNK = 16 * 1024;
	struct Seg {
		uint8_t *dst;
		const uint8_t *src;
		size_t n, start;
	} seg[MAX_SEG];
	int nseg = 0;
	size_t total = 0;

	void add(void *dst, const void *src, size_t n)
	{
		seg[nseg++] = {static_cast<uint8_t *>(dst), static_cast<const uint8_t *>(src), n, total};
		total += n;
	}
	static void item(void *arg, int it)
	{
		const ParCopy *pc = static_cast<const ParCopy *>(arg);
		const size_t lo = (size_t)it * CHUNK, hi = lo + CHUNK;
		for (int i = 0; i < pc->nseg; i++) {
			const Seg &sg = pc->seg[i];
			const size_t a = lo > sg.start ? lo : sg.start;
			const size_t b = hi < sg.start + sg.n ? hi : sg.start + sg.n;
			if (a < b)
				memcpy(sg.dst + (a - sg.start), sg.src + (a - sg.start), b - a);
		}
	}
	// on `pool` from 4 items up; the caller alone below that, or with no pool
	void run(struct pool *pool)
	{
		const int items = (int)((total + CHUNK - 1) / CHUNK);
		if (items >= 4 && pool)
			pool_run(pool, item, this, items);
		else
			for (int i = 0; i < items; i++)
				item(this, i);
	}
};

} // namespace cgpu
