/* SPDX-License-Identifier: GPL-2.0-or-later */
/*
 * The oracle: a CPU restatement of charsiu's quantised-matmul path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product (charsiu_b200/) links,
 * loads or calls this. The tests, the smoke check and the CPU-baseline leg
 * of bench.py use it as the checker that the CUDA path is compared against.
 *
 * Every function restates one reference function in this project's own
 * code and names the reference lines it follows (paths are relative to the
 * charsiu source tree). The restatement is pinned against the reference
 * itself: oracle/Makefile compiles the reference's own sources into
 * oracle/_ref/, and tests/golden/ holds vectors produced by that build.
 */
#ifndef CHARSIU_ORACLE_H
#define CHARSIU_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type numbers, as include/charsiu_llm.h:35-38 fixes them */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q8_0 = 8, ORC_Q6_K = 14 };

/* src/gguf.c:26-55 */
float orc_half_to_float(uint16_t h);

/* Bytes of one row of a q8_0 / q4_0 / q6_K tensor with k columns
 * (src/gguf.c:1166, 1170, 1178). */
uint64_t orc_row_bytes(uint32_t type, uint64_t k);

/*
 * src/gguf.c:829-882: the activation in blocks of 32, one fp32 scale each.
 * q holds nb*32 bytes, d and bs nb floats, nb = (n + 31) / 32.
 */
void orc_act_quantise(const float *x, int n, int8_t *q, float *d, float *bs);

/*
 * src/gguf.c:1149-1171 with dotq_q8_0 (:1098-1107), dotq_q4_0 (:1061-1077)
 * and dotq_q6_K (:1109-1145): rows [row0, row0 + nrows) of y from the integer
 * dots. Returns -1 for a type this restates not (q4_1) or a ragged K.
 */
int orc_matvec(uint32_t type, const void *blocks, uint64_t k, const int8_t *q,
	       const float *d, float *y, uint64_t row0, uint64_t nrows);

/* The integer block dots alone: dots[r * nb + b] for rows [0, n); q8_0 and
 * q4_0 (32-element blocks) only. */
int orc_block_dots(uint32_t type, const void *blocks, uint64_t k, uint64_t n,
		   const int8_t *q, int32_t *dots);

/* src/gguf.c:1217-1278: one row dequantised to fp32 (f32, f16, q8_0, q4_0,
 * q6_K). */
int orc_row_f32(uint32_t type, const void *data, uint64_t k, uint64_t row,
		float *dst);

/*
 * tools/charsiu_matmul.c:41-81 (signed output; int8 weights): the int8
 * matmul with its output stage. a is u8 [m][k], w u8 [n][k], bias i32 [n],
 * out i8 [m][n] row major.
 */
void orc_matmul_i8(unsigned m, unsigned k, unsigned n, const uint8_t *a,
		   const uint8_t *w, const int32_t *bias, float in_scale,
		   float wt_scale, float out_scale, int in_zp, int wt_zp,
		   int out_zp, int8_t *out);

/* ---- the NPU number format (CHARSIU_NPU_QUANT) --------------------------- */

/*
 * npu_tensor_build in its default form (src/npuquant.c:34-296 with none of
 * its CHARSIU_NPU_* experiment switches set: eight bits, one scale a row, no
 * k factor): each row dequantised (gguf_row_f32), amax over it, d = amax /
 * 127, q = lrintf(x * (1 / d)) clamped to [-127, 127]; wsum = the row's sum
 * of q. q [n][k] row major, scale [n], wsum [n] (may be NULL). -1 for a type
 * orc_row_f32 reads not.
 */
int orc_npu_tensor_build(uint32_t type, const void *data, uint64_t k, uint64_t n,
			 int8_t *q, float *scale, int32_t *wsum);

/* charsiu_act_set's single-scale form (src/gguf.c:883-910): d1 = amax / 127,
 * q1[i] = lrintf(x[i] * (1 / d1)) clamped to [-127, 127], zero past n; q1
 * holds nb * 32 bytes. */
void orc_act_quantise_one(const float *x, int n, int8_t *q1, float *d1);

/*
 * y = W x in the NPU format, acc[r] = sum_k q[r][k] * q1[k] (exact int32):
 *   model 0: the device path, src/npudev.c:604-605 (and :707-708):
 *            y[r] = (float)acc * d1 * scale[r], in float, left to right;
 *   model 1: the CPU model, src/npuquant.c:447-544 (one scale a row, no k
 *            factor): y[r] = (float)(((double)acc * scale[r]) * d1).
 */
void orc_npu_matvec(const int8_t *q, const float *scale, uint64_t k, uint64_t n,
		    const int8_t *q1, float d1, int model, float *y);

/* ---- the decode loop (src/llama.c:316-386, 743-868) --------------------- */

struct orc_layer {
	const float *attn_norm, *ffn_norm;            /* f32 [n_embd] */
	const void *w[7];                             /* q k v o gate up down */
	uint32_t type[7];
	const int8_t *nq[7];                          /* NPU format (npu != 0) */
	const float *nscale[7];
};

struct orc_model {
	uint32_t n_embd, n_layer, n_head, n_head_kv, n_ff, n_vocab, head_dim;
	float rms_eps, rope_base;
	const void *tok_embd;  uint32_t tok_type;     /* [n_vocab][n_embd] */
	const void *output;    uint32_t out_type;     /* may be tok_embd */
	const float *out_norm;
	const struct orc_layer *layers;
	/*
	 * 0: every projection and the head through gguf_matvec. 1 or 2: through
	 * the NPU format (CHARSIU_NPU_QUANT, src/llama.c:110-312), the tensors'
	 * npu_tensor_build copies in nq / nscale and out_nq / out_nscale, the
	 * arithmetic of orc_npu_matvec model npu - 1 (1: the device's, 2: the
	 * CPU model's).
	 */
	int npu;
	const int8_t *out_nq;
	const float *out_nscale;
};

struct orc_state;

struct orc_state *orc_state_new(const struct orc_model *m, int n_ctx);
void orc_state_free(struct orc_state *s);
/* one token in, the logit vector out (src/llama.c:743-856) */
const float *orc_forward(struct orc_state *s, int32_t token, int pos);
/* src/llama.c:860-868: the first index of the strict maximum */
int32_t orc_argmax(const float *logits, uint32_t n);
/* greedy decode: prompt, then n_gen tokens into out[]. Returns n_gen or -1. */
int orc_greedy(struct orc_state *s, const int32_t *prompt, int n_prompt,
	       int n_gen, int32_t *out);

#ifdef __cplusplus
}
#endif

#endif
