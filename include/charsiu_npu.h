/* SPDX-License-Identifier: GPL-2.0-or-later */
#ifndef CHARSIU_NPU_GPU_H
#define CHARSIU_NPU_GPU_H

/*
 * charsiu's NPU device layer -- the charsiu_npu_* calls of
 * include/charsiu_llm.h:186-200, implemented by src/npudev.c for the rocket
 * NPU -- over CUDA on a B200. Link this library instead of npudev.c and
 * charsiu's CHARSIU_NPU_QUANT routing (src/llama.c:110-312) runs its
 * projections on the GPU unchanged.
 *
 * The number format is the NPU's (src/npuquant.c): a tensor is npu_tensor_build's
 * int8 copy, one fp32 scale a row; an activation is charsiu_act_set's q1 under
 * ONE scale d1. A matvec returns y[r] = (float)acc[r] * d1 * scale[r] with
 * acc the exact int32 dot -- the arithmetic of src/npudev.c:605 and :710,
 * bit for bit. Conventions are npudev.c's: NULL / -1 means "stay on the CPU for this
 * one", said once on stderr; three slow calls in a row retire the layer; the
 * report says so when nothing ran.
 *
 * The structs are charsiu's own (struct npu_tensor, include/charsiu_llm.h:143-161;
 * struct charsiu_act, :100-119), taken by pointer; the flat forms take plain
 * pointers and sizes.
 */

#include <stddef.h>
#include <stdint.h>

#include "charsiu_gpu.h"

#ifdef __cplusplus
extern "C" {
#endif

struct charsiu_npu;
struct npu_tensor;
struct charsiu_act;

/* charsiu_npu_open (src/npudev.c:140-233): tensors up to max_k columns and max_n
 * rows, at most max_tensors of them. The GPU is CUDA device 0, or the one
 * CHARSIU_GPU_DEVICE names. NULL without a B200. */
CHARSIU_GPU_API struct charsiu_npu *charsiu_npu_open(unsigned max_k, unsigned max_n,
						     unsigned max_tensors);
/* the same on CUDA device `device` */
CHARSIU_GPU_API struct charsiu_npu *charsiu_npu_open_ex(unsigned max_k, unsigned max_n,
							unsigned max_tensors, int device);
CHARSIU_GPU_API void charsiu_npu_close(struct charsiu_npu *g);

/* charsiu_npu_add (src/npudev.c:389-461): copy t's int8 rows and scales to the
 * GPU. The id, or -1: the layer is retired, full, t is wider than opened, or
 * t uses a form the device arithmetic above does not cover (several scales a
 * row, kgroup < k; a k factor, kscale). */
CHARSIU_GPU_API int charsiu_npu_add(struct charsiu_npu *g, const struct npu_tensor *t);

/* charsiu_npu_matvec (src/npudev.c:463-607): y = the tensor times a->q1, a->d1
 * (a->n must be the tensor's K). 0, or -1 (the caller computes it itself). */
CHARSIU_GPU_API int charsiu_npu_matvec(struct charsiu_npu *g, int id, const struct charsiu_act *a,
				       float *y);

/* charsiu_npu_matvec_group (src/npudev.c:621-716): n <= 8 tensors of one K
 * against one activation, one launch; ys[i] gets tensor ids[i]'s y. */
CHARSIU_GPU_API int charsiu_npu_matvec_group(struct charsiu_npu *g, const int *ids, unsigned n,
					     const struct charsiu_act *a, float **ys);

/* charsiu_npu_submits / charsiu_npu_report (src/npudev.c:259-295): calls
 * that ran, and a summary on stderr. */
CHARSIU_GPU_API unsigned long charsiu_npu_submits(const struct charsiu_npu *g);
CHARSIU_GPU_API void charsiu_npu_report(const struct charsiu_npu *g);

/* ---- flat forms ------------------------------------------------------------ */

/* charsiu_npu_add of q [n][k] int8 row major and scale [n]. */
CHARSIU_GPU_API int charsiu_npu_add_flat(struct charsiu_npu *g, const int8_t *q,
					 const float *scale, uint64_t n, uint64_t k,
					 const char *name);
/* charsiu_npu_matvec_group of q1 (k int8) and d1. */
CHARSIU_GPU_API int charsiu_npu_matvec_flat(struct charsiu_npu *g, const int *ids, unsigned n,
					    const int8_t *q1, float d1, unsigned k, float **ys);
/* The same with q1 and every ys[i] in GPU memory, queued on `stream` (a
 * cudaStream_t, NULL for the layer's own) with no host synchronisation; q1
 * holds K rounded up to 16 bytes, zero past K. */
CHARSIU_GPU_API int charsiu_npu_matvec_dev(struct charsiu_npu *g, const int *ids, unsigned n,
					   const int8_t *q1, float d1, float *const *ys,
					   void *stream);
/* the last failure, in words ("" if none); 1 once retired */
CHARSIU_GPU_API const char *charsiu_npu_error(const struct charsiu_npu *g);
CHARSIU_GPU_API int charsiu_npu_dead(const struct charsiu_npu *g);

#ifdef __cplusplus
}
#endif

#endif
