// SPDX-License-Identifier: GPL-2.0-or-later
// What the decode step (decoder.cu) reads of a GPU layer beyond the C ABI.
// Hidden symbols of the library, not part of include/charsiu_gpu.h.
#pragma once

#include <cstdint>

struct charsiu_gpu;

namespace cgpu {

int layer_device(const charsiu_gpu *g);
bool layer_no_pdl(const charsiu_gpu *g);
bool layer_whole(const charsiu_gpu *g);
bool layer_tensor(const charsiu_gpu *g, int id, uint64_t *k, uint64_t *rows, uint32_t *type);
void layer_whine(charsiu_gpu *g, const char *why);

} // namespace cgpu
