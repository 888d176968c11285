// SPDX-License-Identifier: GPL-2.0-or-later
// CPU check of cgpu::ParCopy (charsiu_b200/csrc/host_copy.h), built and run by
// tests/test_host_copy.py: random sets of up to eight segments, sizes across
// the 16 KB item edges (0, 1, an item less or more one, several hundred KB),
// copied by the caller alone or on host/pool.c pools of 1, 3 and 7 workers.
// Every destination must equal its source and the guard bytes around it must
// be untouched. Prints "ok <cases>" and exits 0, or the first bad case and 1.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <vector>

#include "host_copy.h"

namespace {

constexpr size_t GUARD = 64;
constexpr uint8_t GUARD_BYTE = 0xa5;

size_t pick_size(std::mt19937_64 &rng)
{
	static const size_t edges[] = {0, 1, 15, 16, cgpu::ParCopy::CHUNK - 1, cgpu::ParCopy::CHUNK,
				       cgpu::ParCopy::CHUNK + 1, 3 * cgpu::ParCopy::CHUNK + 7};
	switch (rng() % 3) {
	case 0:
		return edges[rng() % (sizeof(edges) / sizeof(edges[0]))];
	case 1:
		return rng() % (4 * cgpu::ParCopy::CHUNK);
	default:
		return rng() % (300 * 1024);
	}
}

} // namespace

int main()
{
	std::mt19937_64 rng(20261202);
	struct pool *pools[4] = {nullptr, pool_new(1), pool_new(3), pool_new(7)};
	int cases = 0;
	for (int trial = 0; trial < 400; trial++) {
		const int nseg = 1 + (int)(rng() % cgpu::ParCopy::MAX_SEG);
		std::vector<std::vector<uint8_t>> src(nseg), dst(nseg);
		cgpu::ParCopy pc;
		size_t total = 0;
		for (int i = 0; i < nseg; i++) {
			const size_t n = pick_size(rng);
			src[i].resize(n + 1);
			for (auto &b : src[i])
				b = (uint8_t)rng();
			dst[i].assign(n + 2 * GUARD, GUARD_BYTE);
			pc.add(dst[i].data() + GUARD, src[i].data(), n);
			total += n;
		}
		if (pc.total != total) {
			std::printf("trial %d: total %zu, segments sum to %zu\n", trial, pc.total, total);
			return 1;
		}
		struct pool *p = pools[trial % 4];
		pc.run(p);
		cases++;
		for (int i = 0; i < nseg; i++) {
			const size_t n = src[i].size() - 1;
			if (std::memcmp(dst[i].data() + GUARD, src[i].data(), n) != 0) {
				std::printf("trial %d (%d segments, pool %d): segment %d of %zu bytes differs\n",
					    trial, nseg, trial % 4, i, n);
				return 1;
			}
			for (size_t j = 0; j < GUARD; j++)
				if (dst[i][j] != GUARD_BYTE || dst[i][GUARD + n + j] != GUARD_BYTE) {
					std::printf("trial %d: segment %d of %zu bytes wrote outside itself\n",
						    trial, i, n);
					return 1;
				}
		}
	}
	for (struct pool *p : pools)
		pool_free(p);
	std::printf("ok %d\n", cases);
	return 0;
}
