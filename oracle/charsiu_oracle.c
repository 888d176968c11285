// SPDX-License-Identifier: GPL-2.0-or-later
/*
 * The oracle: charsiu's quantised-matmul path restated on the CPU.
 *
 * TEST INFRASTRUCTURE ONLY -- the checker, never the thing measured or
 * shipped. See charsiu_oracle.h for what each function restates.
 *
 * Built with gcc -O2 -std=c11 like the reference (its Makefile:8), which
 * leaves floating-point contraction off, so every multiply and add below
 * rounds on its own exactly as the reference's portable kernels do.
 */
#define _POSIX_C_SOURCE 200809L

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "charsiu_oracle.h"

/* ---- fp16 (src/gguf.c:26-55) ------------------------------------------- */

float orc_half_to_float(uint16_t h)
{
	uint32_t sign = (uint32_t)(h >> 15) << 31;
	uint32_t exp = (h >> 10) & 0x1fu;
	uint32_t man = h & 0x3ffu;
	uint32_t bits;
	float f;

	if (exp == 0x1f) {
		bits = sign | 0x7f800000u | (man << 13);
	} else if (exp) {
		bits = sign | ((exp + 112u) << 23) | (man << 13);
	} else if (!man) {
		bits = sign;
	} else {
		/* a subnormal half is a normal float: shift the leading one up */
		int shift = 0;

		while (!(man & 0x400u)) {
			man <<= 1;
			shift++;
		}
		bits = sign | ((uint32_t)(113 - shift) << 23) | ((man & 0x3ffu) << 13);
	}
	memcpy(&f, &bits, 4);
	return f;
}

static uint16_t rd16(const uint8_t *p)
{
	return (uint16_t)(p[0] | (p[1] << 8));
}

uint64_t orc_row_bytes(uint32_t type, uint64_t k)
{
	switch (type) {
	case ORC_Q8_0: return k / 32 * 34;
	case ORC_Q4_0: return k / 32 * 18;
	case ORC_Q6_K: return k / 256 * 210;
	case ORC_F32:  return k * 4;
	case ORC_F16:  return k * 2;
	default:       return 0;
	}
}

/* ---- the activation (src/gguf.c:829-882) -------------------------------- */

void orc_act_quantise(const float *x, int n, int8_t *q, float *d, float *bs)
{
	int nb = (n + 31) / 32;

	for (int b = 0; b < nb; b++) {
		float amax = 0.0f, sum = 0.0f, scale, inv;

		for (int j = 0; j < 32; j++) {
			int i = b * 32 + j;
			float v = i < n ? x[i] : 0.0f;
			float mag = v < 0.0f ? -v : v;

			if (mag > amax)
				amax = mag;
			sum += v;
		}
		scale = amax / 127.0f;
		inv = scale != 0.0f ? 1.0f / scale : 0.0f;
		d[b] = scale;
		if (bs)
			bs[b] = sum;
		/* ties to even (lrintf), gguf.c:871-879 */
		for (int j = 0; j < 32; j++) {
			int i = b * 32 + j;
			float v = i < n ? x[i] : 0.0f;

			q[i] = (int8_t)lrintf(v * inv);
		}
	}
}

/* ---- the integer block dots (src/gguf.c:1052-1107) --------------------- */

static int32_t dot_block_q8(const uint8_t *blk, const int8_t *xq)
{
	const int8_t *w = (const int8_t *)(blk + 2);
	int32_t t = 0;

	for (int j = 0; j < 32; j++)
		t += (int32_t)w[j] * (int32_t)xq[j];
	return t;
}

static int32_t dot_block_q4(const uint8_t *blk, const int8_t *xq)
{
	const uint8_t *nib = blk + 2;
	int32_t t = 0;

	/* byte j: low nibble is element j, high nibble element j + 16 */
	for (int j = 0; j < 16; j++) {
		t += (int32_t)((nib[j] & 0x0f) - 8) * xq[j];
		t += (int32_t)((nib[j] >> 4) - 8) * xq[j + 16];
	}
	return t;
}

static float dot_row(uint32_t type, const uint8_t *row, const int8_t *q,
		     const float *d, uint64_t nb)
{
	unsigned bsz = type == ORC_Q8_0 ? 34 : 18;
	float s = 0.0f;

	for (uint64_t b = 0; b < nb; b++) {
		const uint8_t *blk = row + b * bsz;
		int32_t t = type == ORC_Q8_0 ? dot_block_q8(blk, q + b * 32)
					     : dot_block_q4(blk, q + b * 32);
		/* (d_w * d_a) * t, then the add: left to right, two roundings */
		float scale = orc_half_to_float(rd16(blk)) * d[b];

		s += scale * (float)t;
	}
	return s;
}

/*
 * q6_K (src/gguf.c:449-454 for the 210-byte super-block, :1109-1145 for the
 * integer dot). A super-block holds 256 weights as two halves of 128; in half
 * h, byte l (0..63) of ql and byte l (0..31) of qh give four 6-bit weights
 * (low nibble of ql[l] / ql[l + 32], high nibble of the same, each with two
 * bits of qh[l] above it), minus 32. Every 16 weights have one int8 scale; an
 * activation block (32) covers two such runs, so each run's integer dot is
 * scaled by ((d * scale) * d_a) and added to the row's sum in the order
 * (super-block, half, run pair g, run k).
 */
static int q6_weight(const uint8_t *ql, const uint8_t *qh, unsigned k, unsigned l)
{
	unsigned lo = (k & 1) ? ql[l + 32] : ql[l];
	unsigned nib = (k & 2) ? lo >> 4 : lo & 0x0f;
	unsigned hi = (qh[l] >> (2 * k)) & 3;

	return (int)(nib | (hi << 4)) - 32;
}

static float dot_row_q6k(const uint8_t *row, const int8_t *q, const float *d, uint64_t nsb)
{
	float s = 0.0f;

	for (uint64_t i = 0; i < nsb; i++) {
		const uint8_t *sb = row + i * 210;
		float dd = orc_half_to_float(rd16(sb + 208));

		for (unsigned h = 0; h < 2; h++) {
			const uint8_t *ql = sb + h * 64, *qh = sb + 128 + h * 32;
			const int8_t *sc = (const int8_t *)(sb + 192) + h * 8;
			const int8_t *xq = q + i * 256 + h * 128;
			const float *xd = d + i * 8 + h * 4;

			for (unsigned g = 0; g < 2; g++)
				for (unsigned k = 0; k < 4; k++) {
					int32_t t = 0;

					for (unsigned j = 0; j < 16; j++) {
						unsigned l = g * 16 + j;

						t += q6_weight(ql, qh, k, l) * xq[k * 32 + l];
					}
					s += dd * (float)sc[g + 2 * k] * xd[k] * (float)t;
				}
		}
	}
	return s;
}

int orc_matvec(uint32_t type, const void *blocks, uint64_t k, const int8_t *q,
	       const float *d, float *y, uint64_t row0, uint64_t nrows)
{
	const uint8_t *base = blocks;
	uint64_t rb = orc_row_bytes(type, k);

	if (type == ORC_Q6_K) {
		if (k % 256)
			return -1;
		for (uint64_t r = row0; r < row0 + nrows; r++)
			y[r] = dot_row_q6k(base + r * rb, q, d, k / 256);
		return 0;
	}
	if ((type != ORC_Q8_0 && type != ORC_Q4_0) || k % 32)
		return -1;
	for (uint64_t r = row0; r < row0 + nrows; r++)
		y[r] = dot_row(type, base + r * rb, q, d, k / 32);
	return 0;
}

int orc_block_dots(uint32_t type, const void *blocks, uint64_t k, uint64_t n,
		   const int8_t *q, int32_t *dots)
{
	const uint8_t *base = blocks;
	uint64_t nb = k / 32, rb = orc_row_bytes(type, k);
	unsigned bsz = type == ORC_Q8_0 ? 34 : 18;

	if ((type != ORC_Q8_0 && type != ORC_Q4_0) || k % 32)
		return -1;
	for (uint64_t r = 0; r < n; r++)
		for (uint64_t b = 0; b < nb; b++) {
			const uint8_t *blk = base + r * rb + b * bsz;

			dots[r * nb + b] = type == ORC_Q8_0
				? dot_block_q8(blk, q + b * 32)
				: dot_block_q4(blk, q + b * 32);
		}
	return 0;
}

/* ---- one row to fp32 (src/gguf.c:1217-1256) ----------------------------- */

int orc_row_f32(uint32_t type, const void *data, uint64_t k, uint64_t row,
		float *dst)
{
	const uint8_t *p = (const uint8_t *)data + row * orc_row_bytes(type, k);

	switch (type) {
	case ORC_F32:
		memcpy(dst, p, k * 4);
		return 0;
	case ORC_F16:
		for (uint64_t i = 0; i < k; i++)
			dst[i] = orc_half_to_float(rd16(p + 2 * i));
		return 0;
	case ORC_Q8_0:
		for (uint64_t b = 0; b < k / 32; b++) {
			const uint8_t *blk = p + b * 34;
			float dd = orc_half_to_float(rd16(blk));

			for (int j = 0; j < 32; j++)
				dst[b * 32 + j] = dd * (float)(int8_t)blk[2 + j];
		}
		return 0;
	case ORC_Q4_0:
		for (uint64_t b = 0; b < k / 32; b++) {
			const uint8_t *blk = p + b * 18;
			float dd = orc_half_to_float(rd16(blk));

			for (int j = 0; j < 16; j++) {
				dst[b * 32 + j] = dd * (float)((blk[2 + j] & 0x0f) - 8);
				dst[b * 32 + j + 16] = dd * (float)((blk[2 + j] >> 4) - 8);
			}
		}
		return 0;
	case ORC_Q6_K:
		/* (d * scale) * q, the order of src/gguf.c:457-479 */
		for (uint64_t i = 0; i < k / 256; i++) {
			const uint8_t *sb = p + i * 210;
			float dd = orc_half_to_float(rd16(sb + 208));

			for (unsigned h = 0; h < 2; h++) {
				const uint8_t *ql = sb + h * 64, *qh = sb + 128 + h * 32;
				const int8_t *sc = (const int8_t *)(sb + 192) + h * 8;
				float *out = dst + i * 256 + h * 128;

				for (unsigned l = 0; l < 32; l++)
					for (unsigned kk = 0; kk < 4; kk++)
						out[kk * 32 + l] = dd * (float)sc[l / 16 + 2 * kk] *
								   (float)q6_weight(ql, qh, kk, l);
			}
		}
		return 0;
	default:
		return -1;
	}
}

/* ---- the NPU number format (src/npuquant.c, src/npudev.c, src/gguf.c) ---- */

int orc_npu_tensor_build(uint32_t type, const void *data, uint64_t k, uint64_t n,
			 int8_t *q, float *scale, int32_t *wsum)
{
	float *row = malloc(k * sizeof(float));

	if (!row)
		return -1;
	for (uint64_t r = 0; r < n; r++) {
		float amax = 0.0f, d, id;
		int32_t sum = 0;

		if (orc_row_f32(type, data, k, r, row) < 0) {
			free(row);
			return -1;
		}
		for (uint64_t i = 0; i < k; i++) {
			float a = fabsf(row[i]);

			if (a > amax)
				amax = a;
		}
		/* symmetric over [-127, 127] (src/npuquant.c:196-201) */
		d = amax / 127.0f;
		id = d != 0.0f ? 1.0f / d : 0.0f;
		scale[r] = d;
		for (uint64_t i = 0; i < k; i++) {
			int v = (int)lrintf(row[i] * id);

			if (v > 127)
				v = 127;
			if (v < -127)
				v = -127;
			q[r * k + i] = (int8_t)v;
			sum += v;
		}
		if (wsum)
			wsum[r] = sum;
	}
	free(row);
	return 0;
}

void orc_act_quantise_one(const float *x, int n, int8_t *q1, float *d1)
{
	int nb = (n + 31) / 32;
	float amax = 0.0f, d, id;

	for (int i = 0; i < n; i++) {
		float av = x[i] < 0.0f ? -x[i] : x[i];

		if (av > amax)
			amax = av;
	}
	d = amax / 127.0f;
	id = d != 0.0f ? 1.0f / d : 0.0f;
	*d1 = d;
	for (int i = 0; i < nb * 32; i++) {
		int v = i < n ? (int)lrintf(x[i] * id) : 0;

		if (v > 127)
			v = 127;
		if (v < -127)
			v = -127;
		q1[i] = (int8_t)v;
	}
}

void orc_npu_matvec(const int8_t *q, const float *scale, uint64_t k, uint64_t n,
		    const int8_t *q1, float d1, int model, float *y)
{
	for (uint64_t r = 0; r < n; r++) {
		const int8_t *w = q + r * k;
		int32_t acc = 0;

		for (uint64_t i = 0; i < k; i++)
			acc += (int32_t)w[i] * (int32_t)q1[i];
		if (model == 0) {
			y[r] = (float)acc * d1 * scale[r];
		} else {
			double a = 0.0;

			a += (double)acc * scale[r];
			y[r] = (float)(a * d1);
		}
	}
}

/* ---- int8 matmul + output stage (tools/charsiu_matmul.c:41-81) ---------- */

void orc_matmul_i8(unsigned m, unsigned k, unsigned n, const uint8_t *a,
		   const uint8_t *w, const int32_t *bias, float in_scale,
		   float wt_scale, float out_scale, int in_zp, int wt_zp,
		   int out_zp, int8_t *out)
{
	float mult = in_scale * wt_scale / out_scale;

	for (unsigned i = 0; i < m; i++)
		for (unsigned c = 0; c < n; c++) {
			int64_t acc = bias[c];
			float v;

			for (unsigned j = 0; j < k; j++)
				acc += (int64_t)((int)a[(size_t)i * k + j] - in_zp) *
				       ((int)w[(size_t)c * k + j] - wt_zp);
			/* half up is floor(v + 0.5), not a cast */
			v = (float)acc * mult + (float)out_zp;
			v = floorf(v + 0.5f);
			if (v < -128.0f)
				v = -128.0f;
			if (v > 127.0f)
				v = 127.0f;
			out[(size_t)i * n + c] = (int8_t)(int)v;
		}
}

/* ---- the decode loop (src/llama.c:316-386, 743-868) --------------------- */

struct orc_state {
	const struct orc_model *m;
	int n_ctx;
	float *kcache, *vcache;
	float *x, *xb, *xb2, *hb, *hb2, *q, *k, *v, *att, *logits;
	int8_t *aq, *aq1;
	float *ad, ad1;
};

struct orc_state *orc_state_new(const struct orc_model *m, int n_ctx)
{
	struct orc_state *s = calloc(1, sizeof(*s));
	size_t kvn = (size_t)m->n_layer * (size_t)n_ctx * m->n_head_kv * m->head_dim;
	uint32_t widest = m->n_embd > m->n_ff ? m->n_embd : m->n_ff;

	if (!s)
		return NULL;
	s->m = m;
	s->n_ctx = n_ctx;
	s->kcache = calloc(kvn, sizeof(float));
	s->vcache = calloc(kvn, sizeof(float));
	s->x = calloc(m->n_embd, sizeof(float));
	s->xb = calloc(m->n_embd, sizeof(float));
	s->xb2 = calloc(m->n_embd, sizeof(float));
	s->hb = calloc(m->n_ff, sizeof(float));
	s->hb2 = calloc(m->n_ff, sizeof(float));
	s->q = calloc((size_t)m->n_head * m->head_dim, sizeof(float));
	s->k = calloc((size_t)m->n_head_kv * m->head_dim, sizeof(float));
	s->v = calloc((size_t)m->n_head_kv * m->head_dim, sizeof(float));
	s->att = calloc((size_t)m->n_head * n_ctx, sizeof(float));
	s->logits = calloc(m->n_vocab, sizeof(float));
	s->aq = calloc((size_t)(widest + 31) / 32 * 32, 1);
	s->ad = calloc((size_t)(widest + 31) / 32, sizeof(float));
	s->aq1 = calloc((size_t)(widest + 31) / 32 * 32, 1);
	if (!s->aq1 || !s->kcache || !s->vcache || !s->x || !s->xb || !s->xb2 || !s->hb ||
	    !s->hb2 || !s->q || !s->k || !s->v || !s->att || !s->logits ||
	    !s->aq || !s->ad) {
		orc_state_free(s);
		return NULL;
	}
	return s;
}

void orc_state_free(struct orc_state *s)
{
	if (!s)
		return;
	free(s->kcache); free(s->vcache);
	free(s->x); free(s->xb); free(s->xb2); free(s->hb); free(s->hb2);
	free(s->q); free(s->k); free(s->v); free(s->att); free(s->logits);
	free(s->aq); free(s->ad); free(s->aq1);
	free(s);
}

/* llama.c:316-343 */
static void rmsnorm(float *out, const float *x, const float *g, uint32_t n,
		    float eps)
{
	float ss = 0.0f, scale;

	for (uint32_t i = 0; i < n; i++)
		ss += x[i] * x[i];
	scale = 1.0f / sqrtf(ss / (float)n + eps);
	for (uint32_t i = 0; i < n; i++)
		out[i] = x[i] * scale * g[i];
}

/* llama.c:345-358 */
static void softmax(float *x, int n)
{
	float mx = x[0], sum = 0.0f;

	for (int i = 1; i < n; i++)
		if (x[i] > mx)
			mx = x[i];
	for (int i = 0; i < n; i++) {
		x[i] = expf(x[i] - mx);
		sum += x[i];
	}
	for (int i = 0; i < n; i++)
		x[i] /= sum;
}

/* llama.c:366-386: interleaved pairs (2i, 2i+1), no frequency factors */
static void rope(float *v, uint32_t nheads, uint32_t hd, int pos, float base)
{
	for (uint32_t h = 0; h < nheads; h++) {
		float *p = v + h * hd;

		for (uint32_t i = 0; i < hd / 2; i++) {
			float theta = (float)pos * powf(base, -2.0f * (float)i / (float)hd);
			float c = cosf(theta), sn = sinf(theta);
			float x0 = p[2 * i], x1 = p[2 * i + 1];

			p[2 * i] = x0 * c - x1 * sn;
			p[2 * i + 1] = x0 * sn + x1 * c;
		}
	}
}

/* quantise once, then each projection of it (llama.c:178-183, 215-248); in
 * the NPU format the single-scale activation and the tensor's npu copy
 * (llama.c:255-290) */
static void project_nq(struct orc_state *s, uint32_t kdim, const int8_t *nq,
		       const float *nscale, uint32_t ndim, float *y)
{
	orc_npu_matvec(nq, nscale, kdim, ndim, s->aq1, s->ad1, s->m->npu - 1, y);
}

static void project(struct orc_state *s, const float *x, uint32_t kdim,
		    const void *w, uint32_t type, uint32_t ndim, float *y,
		    const int8_t *nq, const float *nscale)
{
	orc_act_quantise(x, (int)kdim, s->aq, s->ad, NULL);
	if (s->m->npu) {
		orc_act_quantise_one(x, (int)kdim, s->aq1, &s->ad1);
		project_nq(s, kdim, nq, nscale, ndim, y);
		return;
	}
	orc_matvec(type, w, kdim, s->aq, s->ad, y, 0, ndim);
}

static void project_again(struct orc_state *s, uint32_t kdim, const void *w,
			  uint32_t type, uint32_t ndim, float *y,
			  const int8_t *nq, const float *nscale)
{
	if (s->m->npu) {
		project_nq(s, kdim, nq, nscale, ndim, y);
		return;
	}
	orc_matvec(type, w, kdim, s->aq, s->ad, y, 0, ndim);
}

const float *orc_forward(struct orc_state *s, int32_t token, int pos)
{
	const struct orc_model *m = s->m;
	uint32_t hd = m->head_dim, kvdim = m->n_head_kv * hd;
	uint32_t gqa = m->n_head / m->n_head_kv;
	float scale = 1.0f / sqrtf((float)hd);

	if (pos >= s->n_ctx)
		return NULL;
	orc_row_f32(m->tok_type, m->tok_embd, m->n_embd, (uint64_t)token, s->x);

	for (uint32_t l = 0; l < m->n_layer; l++) {
		const struct orc_layer *L = &m->layers[l];
		float *kc = s->kcache + ((size_t)l * s->n_ctx + pos) * kvdim;
		float *vc = s->vcache + ((size_t)l * s->n_ctx + pos) * kvdim;

		rmsnorm(s->xb, s->x, L->attn_norm, m->n_embd, m->rms_eps);
		project(s, s->xb, m->n_embd, L->w[0], L->type[0], m->n_head * hd, s->q,
			L->nq[0], L->nscale[0]);
		project_again(s, m->n_embd, L->w[1], L->type[1], kvdim, s->k, L->nq[1],
			      L->nscale[1]);
		project_again(s, m->n_embd, L->w[2], L->type[2], kvdim, s->v, L->nq[2],
			      L->nscale[2]);

		rope(s->q, m->n_head, hd, pos, m->rope_base);
		rope(s->k, m->n_head_kv, hd, pos, m->rope_base);
		memcpy(kc, s->k, kvdim * sizeof(float));
		memcpy(vc, s->v, kvdim * sizeof(float));

		/* llama.c:792-818 */
		for (uint32_t h = 0; h < m->n_head; h++) {
			const float *qh = s->q + h * hd;
			float *att = s->att + (size_t)h * s->n_ctx;
			uint32_t kvh = h / gqa;
			float *out = s->xb + h * hd;

			for (int t = 0; t <= pos; t++) {
				const float *kt = s->kcache +
					((size_t)l * s->n_ctx + t) * kvdim + kvh * hd;
				float a = 0.0f;

				for (uint32_t i = 0; i < hd; i++)
					a += qh[i] * kt[i];
				att[t] = a * scale;
			}
			softmax(att, pos + 1);
			memset(out, 0, hd * sizeof(float));
			for (int t = 0; t <= pos; t++) {
				const float *vt = s->vcache +
					((size_t)l * s->n_ctx + t) * kvdim + kvh * hd;
				float a = att[t];

				for (uint32_t i = 0; i < hd; i++)
					out[i] += a * vt[i];
			}
		}

		project(s, s->xb, m->n_embd, L->w[3], L->type[3], m->n_embd, s->xb2,
			L->nq[3], L->nscale[3]);
		for (uint32_t i = 0; i < m->n_embd; i++)
			s->x[i] += s->xb2[i];

		rmsnorm(s->xb, s->x, L->ffn_norm, m->n_embd, m->rms_eps);
		project(s, s->xb, m->n_embd, L->w[4], L->type[4], m->n_ff, s->hb,
			L->nq[4], L->nscale[4]);
		project_again(s, m->n_embd, L->w[5], L->type[5], m->n_ff, s->hb2, L->nq[5],
			      L->nscale[5]);
		for (uint32_t i = 0; i < m->n_ff; i++) {
			float g = s->hb[i];

			g *= 1.0f / (1.0f + expf(-g));
			s->hb[i] = g * s->hb2[i];
		}
		project(s, s->hb, m->n_ff, L->w[6], L->type[6], m->n_embd, s->xb2,
			L->nq[6], L->nscale[6]);
		for (uint32_t i = 0; i < m->n_embd; i++)
			s->x[i] += s->xb2[i];
	}

	rmsnorm(s->xb, s->x, m->out_norm, m->n_embd, m->rms_eps);
	project(s, s->xb, m->n_embd, m->output, m->out_type, m->n_vocab, s->logits,
		m->out_nq, m->out_nscale);
	return s->logits;
}

int32_t orc_argmax(const float *logits, uint32_t n)
{
	int32_t best = 0;

	for (uint32_t i = 1; i < n; i++)
		if (logits[i] > logits[best])
			best = (int32_t)i;
	return best;
}

int orc_greedy(struct orc_state *s, const int32_t *prompt, int n_prompt,
	       int n_gen, int32_t *out)
{
	const float *logits = NULL;
	int pos = 0;

	for (int i = 0; i < n_prompt; i++)
		if (!(logits = orc_forward(s, prompt[i], pos++)))
			return -1;
	for (int i = 0; i < n_gen; i++) {
		out[i] = orc_argmax(logits, s->m->n_vocab);
		if (i + 1 < n_gen && !(logits = orc_forward(s, out[i], pos++)))
			return -1;
	}
	return n_gen;
}
