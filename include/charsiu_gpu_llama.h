/* SPDX-License-Identifier: GPL-2.0-or-later */
#ifndef CHARSIU_GPU_LLAMA_H
#define CHARSIU_GPU_LLAMA_H

/*
 * charsiu's decode loop with every projection routed to the GPU layer.
 *
 * This is what the reference's src/llama.c does once its matvec routing
 * (src/llama.c:178-312) sends the 112 projections and the output head to
 * charsiu_gpu_* instead of the pool: the same GGUF model, the same CPU
 * rmsnorm / rope / attention / SwiGLU in the same float order, the activation
 * quantised once per matvec exactly as charsiu_act_set does, and q/k/v and
 * gate/up sent as one group call each. Its logits are bit-identical to
 * llama_forward's. A failed GPU call is an error here (NULL / -1), never a
 * silent CPU result.
 */

#include <stdint.h>

#include "charsiu_gpu.h"

#ifdef __cplusplus
extern "C" {
#endif

struct charsiu_gpu_llama;

/* llama_load + llama_state_new (include/charsiu_llm.h:298-301): map the
 * GGUF, open the GPU layer on `device`, upload and repack every projection
 * and the head. n_ctx <= 0: the training context capped at 4096
 * (src/llama.c:530-532). NULL on failure. */
CHARSIU_GPU_API struct charsiu_gpu_llama *charsiu_gpu_llama_open(const char *gguf_path, int n_ctx,
						 int device);
CHARSIU_GPU_API void charsiu_gpu_llama_close(struct charsiu_gpu_llama *m);

/* Run every later forward on the device (on != 0: charsiu_gpu_decoder_*,
 * include/charsiu_gpu.h -- the rmsnorm, RoPE, attention, SiLU, residuals and
 * argmax as well as the projections, one CUDA graph a token, the same logits
 * bit for bit) or with the CPU steps here (0, the default: the reference's
 * loop with only its matvecs routed). The first switch on builds the device
 * step, which keeps its own KV cache: switch before the first token. The
 * environment variable CHARSIU_GPU_RESIDENT=1 switches on at open. 0 on
 * success; -1 if the device step cannot be built (the mode is unchanged). */
CHARSIU_GPU_API int charsiu_gpu_llama_set_resident(struct charsiu_gpu_llama *m, int on);

/* llama_forward (include/charsiu_llm.h:307): one token at `pos`, the logits
 * out (n_vocab floats, valid until the next call). NULL on failure. */
CHARSIU_GPU_API const float *charsiu_gpu_llama_forward(struct charsiu_gpu_llama *m, int32_t token, int pos);

/* llama_argmax (include/charsiu_llm.h:310): the first index of the maximum */
CHARSIU_GPU_API int32_t charsiu_gpu_llama_argmax(const float *logits, uint32_t n);

/* Greedy decode as tools/charsiu_run.c:220-317 runs it: the prompt, then
 * n_gen tokens into out. If logits is given, the logits each generated token
 * was chosen from are copied to logits[i * n_vocab]. *gen_ms gets the time of
 * the generation loop. Returns n_gen, or -1. */
CHARSIU_GPU_API int charsiu_gpu_llama_greedy(struct charsiu_gpu_llama *m, const int32_t *prompt, int n_prompt,
			     int n_gen, int32_t *out, float *logits, double *gen_ms);

/* llama_stages_report (src/llama.c:684-739): the mean ms a token of each
 * of the forward pass's 14 stages into ms_per_token[0..n), since open or the
 * last reset. Returns the number of stages. CHARSIU_STAGES=1 also prints the
 * table at close. */
CHARSIU_GPU_API int charsiu_gpu_llama_stages(struct charsiu_gpu_llama *m, double *ms_per_token,
					     int n, int reset);
CHARSIU_GPU_API const char *charsiu_gpu_llama_stage_name(int i);

CHARSIU_GPU_API uint32_t charsiu_gpu_llama_vocab(const struct charsiu_gpu_llama *m);
/* the device layer the model runs on (for its report and counters) */
CHARSIU_GPU_API struct charsiu_gpu *charsiu_gpu_llama_layer(struct charsiu_gpu_llama *m);
/* the NPU-format layer when the model was opened with CHARSIU_NPU_QUANT=1
 * (every projection and the head in charsiu's NPU number format through
 * charsiu_npu_*, include/charsiu_npu.h, as src/llama.c:110-312 routes them);
 * else NULL */
CHARSIU_GPU_API struct charsiu_npu *charsiu_gpu_llama_npu(struct charsiu_gpu_llama *m);
/* the device step, once charsiu_gpu_llama_set_resident has built it; else NULL */
CHARSIU_GPU_API struct charsiu_gpu_decoder *charsiu_gpu_llama_decoder(struct charsiu_gpu_llama *m);

#ifdef __cplusplus
}
#endif

#endif
