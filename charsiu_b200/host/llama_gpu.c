// SPDX-License-Identifier: GPL-2.0-or-later
/*
 * charsiu's decode loop with the projections on the GPU layer.
 *
 * The CPU steps restate src/llama.c:316-386 and 743-856 operation for
 * operation (compiled with -std=c11 -ffp-contract=off, so each float op rounds
 * on its own as in the reference); the activation quantiser restates
 * charsiu_act_set (src/gguf.c:852-881). Every matmul goes through the C ABI of
 * include/charsiu_gpu.h with host buffers, exactly as a routed llama.c would
 * call it, so this file is also the end-to-end measurement of that boundary.
 */
#define _POSIX_C_SOURCE 200809L

#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include "charsiu_gpu_llama.h"
#include "charsiu_npu.h"
#include "pool.h"

/* internal to the library (csrc/charsiu_gpu.cu): lend the layer this loop's
 * host threads for its large copies; NULL takes them back */
void charsiu_gpu_lend_pool(struct charsiu_gpu *g, struct pool *p);
void charsiu_npu_lend_pool(struct charsiu_npu *g, struct pool *p);

#define API

enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q6_K = 14 };

/* ---- a GGUF v2/v3 reader (the format src/gguf.c:207-358 reads) ----------- */

struct gt {
	char name[80];
	uint64_t ne[4];
	uint32_t n_dims, type;
	uint64_t offset;
	const uint8_t *data;
};

struct gfile {
	int fd;
	const uint8_t *map;
	size_t size;
	struct gt *t;
	uint64_t nt;
	/* the keys the model needs */
	char arch[64];
	uint32_t u[16];
	int have[16];
	float f[4];
	int have_f[4];
	uint64_t n_tokens;
};

enum { K_EMBD, K_LAYERS, K_HEAD, K_HEAD_KV, K_FF, K_CTX, K_ROPE_DIM, K_ALIGN, K_NU };
enum { F_EPS, F_BASE, K_NF };

struct cur {
	const uint8_t *p, *end;
	int bad;
};

static int take(struct cur *c, void *dst, size_t n)
{
	if (c->bad || (size_t)(c->end - c->p) < n) {
		c->bad = 1;
		return -1;
	}
	if (dst)
		memcpy(dst, c->p, n);
	c->p += n;
	return 0;
}

static uint64_t u64(struct cur *c)
{
	uint64_t v = 0;
	take(c, &v, 8);
	return v;
}

static uint32_t u32(struct cur *c)
{
	uint32_t v = 0;
	take(c, &v, 4);
	return v;
}

static const char *str(struct cur *c, uint64_t *len)
{
	uint64_t n = u64(c);
	const char *s = (const char *)c->p;

	if (c->bad || (uint64_t)(c->end - c->p) < n) {
		c->bad = 1;
		*len = 0;
		return "";
	}
	c->p += n;
	*len = n;
	return s;
}

static size_t vsize(uint32_t t)
{
	static const size_t w[13] = { 1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8 };
	return t < 13 ? w[t] : 0;
}

static int key_is(const char *k, uint64_t kl, const char *arch, const char *suffix)
{
	char full[128];

	snprintf(full, sizeof(full), "%s.%s", arch, suffix);
	return kl == strlen(full) && !memcmp(k, full, kl);
}

static uint64_t tensor_bytes(uint32_t type, const uint64_t ne[4])
{
	uint64_t n = ne[0] * ne[1] * ne[2] * ne[3];

	switch (type) {
	case T_F32: return n * 4;
	case T_F16: return n * 2;
	case T_Q8_0: return n / 32 * 34;
	case T_Q4_0: return n / 32 * 18;
	case T_Q6_K: return n / 256 * 210;
	default: return 0;
	}
}

static void gclose(struct gfile *g)
{
	free(g->t);
	if (g->map && g->map != MAP_FAILED)
		munmap((void *)g->map, g->size);
	if (g->fd >= 0)
		close(g->fd);
	memset(g, 0, sizeof(*g));
	g->fd = -1;
}

static int gopen(struct gfile *g, const char *path)
{
	static const char *ukeys[K_NU] = {
		"embedding_length", "block_count", "attention.head_count",
		"attention.head_count_kv", "feed_forward_length", "context_length",
		"rope.dimension_count", NULL,
	};
	static const char *fkeys[K_NF] = { "attention.layer_norm_rms_epsilon", "rope.freq_base" };
	struct stat st;
	struct cur c;
	uint64_t nkv, off, align = 32;
	char magic[4];
	uint32_t ver;

	memset(g, 0, sizeof(*g));
	strcpy(g->arch, "llama");
	g->fd = open(path, O_RDONLY);
	if (g->fd < 0 || fstat(g->fd, &st) < 0 || st.st_size < 24) {
		fprintf(stderr, "charsiu: cannot read %s\n", path);
		gclose(g);
		return -1;
	}
	g->size = (size_t)st.st_size;
	g->map = mmap(NULL, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
	if (g->map == MAP_FAILED) {
		gclose(g);
		return -1;
	}
	c.p = g->map;
	c.end = g->map + g->size;
	c.bad = 0;
	take(&c, magic, 4);
	ver = u32(&c);
	if (memcmp(magic, "GGUF", 4) || ver < 2 || ver > 3) {
		fprintf(stderr, "charsiu: %s is not GGUF v2/v3\n", path);
		gclose(g);
		return -1;
	}
	g->nt = u64(&c);
	nkv = u64(&c);
	if (c.bad || g->nt > 100000 || nkv > 100000) {
		gclose(g);
		return -1;
	}
	/* general.architecture comes first in practice, but do not rely on it:
	 * keep the raw arch-prefixed keys and resolve after the walk */
	{
		const uint8_t *kv0 = c.p;

		for (int pass = 0; pass < 2; pass++) {
			c.p = kv0;
			for (uint64_t i = 0; i < nkv && !c.bad; i++) {
				uint64_t kl, sl;
				const char *k = str(&c, &kl);
				uint32_t vt = u32(&c);

				if (vt == 8) {
					const char *s = str(&c, &sl);

					if (pass == 0 && kl == 20 && !memcmp(k, "general.architecture", 20) &&
					    sl < sizeof(g->arch)) {
						memcpy(g->arch, s, sl);
						g->arch[sl] = 0;
					}
				} else if (vt == 9) {
					uint32_t at = u32(&c);
					uint64_t n = u64(&c);

					if (pass == 1 && kl == 21 && !memcmp(k, "tokenizer.ggml.tokens", 21))
						g->n_tokens = n;
					if (vsize(at)) {
						if (n > (uint64_t)(c.end - c.p) / vsize(at)) {
							c.bad = 1;
							break;
						}
						c.p += n * vsize(at);
					} else if (at == 8) {
						for (uint64_t j = 0; j < n && !c.bad; j++)
							str(&c, &sl);
					} else {
						c.bad = 1;
					}
				} else if (vsize(vt)) {
					uint64_t v = 0;
					double fv = 0;

					if (vt == 6) {
						float f32 = 0;

						take(&c, &f32, 4);
						fv = f32;
					} else if (vt == 12) {
						take(&c, &fv, 8);
					} else {
						take(&c, &v, vsize(vt));
					}
					if (pass == 1) {
						for (int j = 0; j < K_NU; j++)
							if (ukeys[j] && key_is(k, kl, g->arch, ukeys[j])) {
								g->u[j] = (uint32_t)v;
								g->have[j] = 1;
							}
						for (int j = 0; j < K_NF; j++)
							if (key_is(k, kl, g->arch, fkeys[j])) {
								g->f[j] = (float)fv;
								g->have_f[j] = 1;
							}
						if (kl == 17 && !memcmp(k, "general.alignment", 17) && v)
							align = v;
					}
				} else {
					c.bad = 1;
				}
			}
		}
	}
	g->t = calloc(g->nt ? g->nt : 1, sizeof(*g->t));
	if (c.bad || !g->t) {
		fprintf(stderr, "charsiu: %s: bad key/value section\n", path);
		gclose(g);
		return -1;
	}
	for (uint64_t i = 0; i < g->nt; i++) {
		struct gt *t = &g->t[i];
		uint64_t nl;
		const char *nm = str(&c, &nl);

		if (nl >= sizeof(t->name))
			nl = sizeof(t->name) - 1;
		memcpy(t->name, nm, nl);
		t->n_dims = u32(&c);
		if (t->n_dims > 4) {
			c.bad = 1;
			break;
		}
		t->ne[0] = t->ne[1] = t->ne[2] = t->ne[3] = 1;
		for (unsigned d = 0; d < t->n_dims; d++)
			t->ne[d] = u64(&c);
		t->type = u32(&c);
		t->offset = u64(&c);
	}
	if (c.bad) {
		gclose(g);
		return -1;
	}
	off = (uint64_t)(c.p - g->map);
	off = (off + align - 1) / align * align;
	for (uint64_t i = 0; i < g->nt; i++) {
		struct gt *t = &g->t[i];

		if (off + t->offset + tensor_bytes(t->type, t->ne) > g->size) {
			fprintf(stderr, "charsiu: %s runs past the end of the file\n", t->name);
			gclose(g);
			return -1;
		}
		t->data = g->map + off + t->offset;
	}
	return 0;
}

static const struct gt *gfind(const struct gfile *g, const char *name)
{
	for (uint64_t i = 0; i < g->nt; i++)
		if (!strcmp(g->t[i].name, name))
			return &g->t[i];
	return NULL;
}

/* ---- the model ------------------------------------------------------------ */

enum { P_Q, P_K, P_V, P_O, P_GATE, P_UP, P_DOWN, P_N };

struct layer {
	const float *attn_norm, *ffn_norm;
	const struct gt *w[P_N];
	int id[P_N];
};

/* where a token's time goes, one clock a step of the forward pass (the
 * same split as the reference's CHARSIU_STAGES, src/llama.c:695-705) */
enum {
	T_EMBED, T_ATTN_NORM, T_QKV, T_ROTARY, T_HEADS, T_OUT_PROJ, T_ADD_ATTN,
	T_FFN_NORM, T_GATE_UP, T_SWIGLU, T_DOWN, T_ADD_FFN, T_OUT_NORM, T_VOCAB,
	T_COUNT
};

static const char *stage_name[T_COUNT] = {
	[T_EMBED] = "embed", [T_ATTN_NORM] = "norm/attn", [T_QKV] = "qkv",
	[T_ROTARY] = "rotary+cache", [T_HEADS] = "attn heads", [T_OUT_PROJ] = "out proj",
	[T_ADD_ATTN] = "add/attn", [T_FFN_NORM] = "norm/ffn", [T_GATE_UP] = "gate|up",
	[T_SWIGLU] = "swiglu", [T_DOWN] = "down", [T_ADD_FFN] = "add/ffn",
	[T_OUT_NORM] = "norm/out", [T_VOCAB] = "vocab head",
};

struct charsiu_gpu_llama {
	struct gfile g;
	double stage_ms[T_COUNT];
	unsigned stage_tok;
	struct charsiu_gpu *dev;
	uint32_t n_embd, n_layer, n_head, n_head_kv, n_ff, n_vocab, hd;
	float eps, base;
	const struct gt *tok, *out;
	const float *out_norm;
	int out_id;
	struct layer *L;
	int n_ctx, nogroup;
	float *kcache, *vcache, *x, *xb, *xb2, *hb, *hb2, *q, *k, *v, *att, *logits;
	float *rope_cs;           /* cos, sin of each pair at the current pos */
	int8_t *aq;
	float *ad;
	struct pool *pool;        /* attention heads and SiLU chunks; NULL = this thread */
	struct charsiu_gpu_decoder *dec;   /* the whole step on the device, when resident */
	int resident;
	/* CHARSIU_NPU_QUANT: every projection and the head in the NPU number
	 * format, through charsiu_npu_* (src/llama.c:110-312) */
	int npu_mode;
	struct charsiu_npu *npu;
	int8_t *aq1;              /* the activation under one scale */
	float ad1;
};

static float half_to_float(uint16_t h)
{
	uint32_t sign = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1f, m = h & 0x3ff, bits;
	float f;

	if (e == 0x1f) {
		bits = sign | 0x7f800000u | (m << 13);
	} else if (e) {
		bits = sign | ((e + 112u) << 23) | (m << 13);
	} else if (!m) {
		bits = sign;
	} else {
		int sh = 0;

		while (!(m & 0x400)) {
			m <<= 1;
			sh++;
		}
		bits = sign | ((uint32_t)(113 - sh) << 23) | ((m & 0x3ff) << 13);
	}
	memcpy(&f, &bits, 4);
	return f;
}

/* one row to fp32: the embedding lookup (src/gguf.c:1217-1256) */
static int row_f32(const struct gt *t, uint64_t row, float *dst)
{
	uint64_t k = t->ne[0];
	const uint8_t *p;

	switch (t->type) {
	case T_F32:
		memcpy(dst, t->data + row * k * 4, k * 4);
		return 0;
	case T_Q8_0:
		p = t->data + row * (k / 32 * 34);
		for (uint64_t b = 0; b < k / 32; b++, p += 34) {
			float d = half_to_float((uint16_t)(p[0] | p[1] << 8));

			for (int j = 0; j < 32; j++)
				dst[b * 32 + j] = d * (float)(int8_t)p[2 + j];
		}
		return 0;
	case T_Q4_0:
		p = t->data + row * (k / 32 * 18);
		for (uint64_t b = 0; b < k / 32; b++, p += 18) {
			float d = half_to_float((uint16_t)(p[0] | p[1] << 8));

			for (int j = 0; j < 16; j++) {
				dst[b * 32 + j] = d * (float)((p[2 + j] & 0x0f) - 8);
				dst[b * 32 + j + 16] = d * (float)((p[2 + j] >> 4) - 8);
			}
		}
		return 0;
	case T_Q6_K:
		/* deq_q6_K (src/gguf.c:457-479): (d * scale) * q, q the 6-bit
		 * weight minus 32 from a nibble of ql and two bits of qh */
		p = t->data + row * (k / 256 * 210);
		for (uint64_t i = 0; i < k / 256; i++, p += 210) {
			float d = half_to_float((uint16_t)(p[208] | p[209] << 8));

			for (unsigned h = 0; h < 2; h++) {
				const uint8_t *ql = p + h * 64, *qh = p + 128 + h * 32;
				const int8_t *sc = (const int8_t *)(p + 192) + h * 8;
				float *y = dst + i * 256 + h * 128;

				for (unsigned l = 0; l < 32; l++)
					for (unsigned r = 0; r < 4; r++) {
						unsigned lo = (r & 1) ? ql[l + 32] : ql[l];
						int q = (int)(((r & 2) ? lo >> 4 : lo & 0x0f) |
							      (((qh[l] >> (2 * r)) & 3u) << 4)) - 32;

						y[r * 32 + l] = d * (float)sc[l / 16 + 2 * r] * (float)q;
					}
			}
		}
		return 0;
	default:
		return -1;
	}
}

#if defined(__SSE2__)
#include <emmintrin.h>

/*
 * One full 32-block of act_set with SSE2, the same values as the scalar form:
 * the block's max |x| is a max (maxps skips a NaN |x| exactly as `av > amax`
 * does, and the order of a max does not matter), d and 1/d are the same
 * scalar divisions, x * (1/d) is the same IEEE multiply, cvtps2dq rounds to
 * nearest even as lrintf (cvtss2si) does, and the int8 is the low byte of the
 * int32 as (int8_t) of lrintf's result is.
 */
static void act_block_sse(const float *x, int8_t *q, float *dout)
{
	const __m128 sign = _mm_set1_ps(-0.0f);
	__m128 v[8], mx = _mm_setzero_ps();
	int32_t iq[32];
	float amax, d, id;

	for (int i = 0; i < 8; i++) {
		v[i] = _mm_loadu_ps(x + 4 * i);
		mx = _mm_max_ps(_mm_andnot_ps(sign, v[i]), mx);
	}
	mx = _mm_max_ps(mx, _mm_shuffle_ps(mx, mx, _MM_SHUFFLE(2, 3, 0, 1)));
	mx = _mm_max_ps(mx, _mm_shuffle_ps(mx, mx, _MM_SHUFFLE(1, 0, 3, 2)));
	amax = _mm_cvtss_f32(mx);
	d = amax / 127.0f;
	id = d != 0.0f ? 1.0f / d : 0.0f;
	*dout = d;
	{
		const __m128 vid = _mm_set1_ps(id);

		for (int i = 0; i < 8; i++)
			_mm_storeu_si128((__m128i *)(iq + 4 * i),
					 _mm_cvtps_epi32(_mm_mul_ps(v[i], vid)));
	}
	for (int j = 0; j < 32; j++)
		q[j] = (int8_t)iq[j];
}
#endif

/* charsiu_act_set's q8_0 form (src/gguf.c:852-881) */
static void act_set(struct charsiu_gpu_llama *m, const float *x, int n)
{
	int nb = (n + 31) / 32;

	for (int b = 0; b < nb; b++) {
#if defined(__SSE2__)
		if (b * 32 + 32 <= n) {
			act_block_sse(x + b * 32, m->aq + b * 32, &m->ad[b]);
			continue;
		}
#endif
		float amax = 0.0f, d, id;

		for (int j = 0; j < 32; j++) {
			float v = b * 32 + j < n ? x[b * 32 + j] : 0.0f;
			float av = v < 0.0f ? -v : v;

			if (av > amax)
				amax = av;
		}
		d = amax / 127.0f;
		id = d != 0.0f ? 1.0f / d : 0.0f;
		m->ad[b] = d;
		for (int j = 0; j < 32; j++) {
			float v = b * 32 + j < n ? x[b * 32 + j] : 0.0f;

			m->aq[b * 32 + j] = (int8_t)lrintf(v * id);
		}
	}
}

/* charsiu_act_set's single-scale form (src/gguf.c:883-910), for the NPU
 * number format: d1 = amax / 127, q1 = lrintf(x * (1 / d1)) clamped to
 * [-127, 127], zero past n */
static void act_q1(struct charsiu_gpu_llama *m, const float *x, int n)
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
	m->ad1 = d;
	for (int i = 0; i < nb * 32; i++) {
		int v = i < n ? (int)lrintf(x[i] * id) : 0;

		if (v > 127)
			v = 127;
		if (v < -127)
			v = -127;
		m->aq1[i] = (int8_t)v;
	}
}

/* npu_tensor_build's default form (src/npuquant.c:34-296: eight bits, one
 * scale a row, no k factor), rows [r0, r1) of t: each row dequantised, amax,
 * d = amax / 127, q = lrintf(x * (1 / d)) clamped to [-127, 127] */
struct npu_build_job {
	const struct gt *t;
	int8_t *q;
	float *scale;
	uint64_t rows_per_item;
	int failed;
};

static void npu_build_rows(void *arg, int item)
{
	struct npu_build_job *j = arg;
	uint64_t k = j->t->ne[0], n = j->t->ne[1];
	uint64_t r0 = (uint64_t)item * j->rows_per_item;
	uint64_t r1 = r0 + j->rows_per_item < n ? r0 + j->rows_per_item : n;
	float *row = malloc(k * sizeof(float));

	if (!row) {
		j->failed = 1;
		return;
	}
	for (uint64_t r = r0; r < r1; r++) {
		float amax = 0.0f, d, id;

		if (row_f32(j->t, r, row)) {
			j->failed = 1;
			break;
		}
		for (uint64_t i = 0; i < k; i++) {
			float a = fabsf(row[i]);

			if (a > amax)
				amax = a;
		}
		d = amax / 127.0f;
		id = d != 0.0f ? 1.0f / d : 0.0f;
		j->scale[r] = d;
		for (uint64_t i = 0; i < k; i++) {
			int v = (int)lrintf(row[i] * id);

			if (v > 127)
				v = 127;
			if (v < -127)
				v = -127;
			j->q[r * k + i] = (int8_t)v;
		}
	}
	free(row);
}

/* the NPU-format copy of t on the GPU layer: its id, or -1 */
static int add_npu(struct charsiu_gpu_llama *m, const struct gt *t)
{
	uint64_t k = t->ne[0], n = t->ne[1];
	struct npu_build_job j = { t, malloc(n * k), malloc(n * sizeof(float)), 64, 0 };
	int id = -1;

	if (j.q && j.scale) {
		pool_run(m->pool, npu_build_rows, &j, (int)((n + j.rows_per_item - 1) / j.rows_per_item));
		if (!j.failed)
			id = charsiu_npu_add_flat(m->npu, j.q, j.scale, n, k, t->name);
	}
	free(j.q);
	free(j.scale);
	return id;
}

static void rmsnorm(float *out, const float *x, const float *gw, uint32_t n, float eps)
{
	float ss = 0.0f, scale;

	for (uint32_t i = 0; i < n; i++)
		ss += x[i] * x[i];
	scale = 1.0f / sqrtf(ss / (float)n + eps);
	for (uint32_t i = 0; i < n; i++)
		out[i] = x[i] * scale * gw[i];
}

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

/* The rotation of pair i at `pos` depends on neither the head nor the layer,
 * so its cos and sin are computed once a token (the same libm calls on the
 * same arguments as src/llama.c:373-379, hence the same values) and applied
 * to every head of every layer. */
static void rope_angles(float *cs, uint32_t hd, int pos, float base)
{
	for (uint32_t i = 0; i < hd / 2; i++) {
		float theta = (float)pos * powf(base, -2.0f * (float)i / (float)hd);

		cs[2 * i] = cosf(theta);
		cs[2 * i + 1] = sinf(theta);
	}
}

static void rope(float *v, uint32_t nheads, uint32_t hd, const float *cs)
{
	for (uint32_t h = 0; h < nheads; h++) {
		float *p = v + h * hd;

		for (uint32_t i = 0; i < hd / 2; i++) {
			float c = cs[2 * i], s = cs[2 * i + 1];
			float x0 = p[2 * i], x1 = p[2 * i + 1];

			p[2 * i] = x0 * c - x1 * s;
			p[2 * i + 1] = x0 * s + x1 * c;
		}
	}
}

/* Build the device-resident step (charsiu_gpu_decoder_*) of this model: the
 * projections already on the layer, the embedding (the head's copy when it is
 * tied, else its own), the norm weights, and RoPE's (cos, sin) for every
 * position, computed here with the same calls as rope_angles. */
static struct charsiu_gpu_decoder *make_decoder(struct charsiu_gpu_llama *m)
{
	struct charsiu_gpu_decoder_desc d;
	struct charsiu_gpu_decoder *dec = NULL;
	int *ids = malloc((size_t)m->n_layer * P_N * sizeof(int));
	const float **an = malloc(m->n_layer * sizeof(*an)), **fn = malloc(m->n_layer * sizeof(*fn));
	float *cs = malloc((size_t)m->n_ctx * m->hd * sizeof(float));
	int embd_id = m->out_id;

	if (!ids || !an || !fn || !cs)
		goto out;
	/* in the NPU format the head is an NPU-layer tensor: the embedding rows
	 * come from a copy of token_embd on the GGML layer */
	if (m->tok != m->out || m->npu_mode) {
		embd_id = charsiu_gpu_add_blocks(m->dev, m->tok->type, m->tok->ne[0], m->tok->ne[1],
						 m->tok->data, m->tok->name);
		if (embd_id < 0)
			goto out;
	}
	for (uint32_t l = 0; l < m->n_layer; l++) {
		for (int p = 0; p < P_N; p++)
			ids[l * P_N + p] = m->L[l].id[p];
		an[l] = m->L[l].attn_norm;
		fn[l] = m->L[l].ffn_norm;
	}
	for (int pos = 0; pos < m->n_ctx; pos++)
		rope_angles(cs + (size_t)pos * m->hd, m->hd, pos, m->base);
	memset(&d, 0, sizeof(d));
	d.n_embd = m->n_embd;
	d.n_layer = m->n_layer;
	d.n_head = m->n_head;
	d.n_head_kv = m->n_head_kv;
	d.n_ff = m->n_ff;
	d.head_dim = m->hd;
	d.n_vocab = m->n_vocab;
	d.n_ctx = (uint32_t)m->n_ctx;
	d.rms_eps = m->eps;
	d.embd_id = embd_id;
	d.head_id = m->out_id;
	d.proj_ids = ids;
	d.attn_norm = an;
	d.ffn_norm = fn;
	d.out_norm = m->out_norm;
	d.rope_cs = cs;
	dec = m->npu_mode ? charsiu_gpu_decoder_new_npu(m->dev, m->npu, &d)
			  : charsiu_gpu_decoder_new(m->dev, &d);
out:
	free(ids);
	free(an);
	free(fn);
	free(cs);
	return dec;
}

API int charsiu_gpu_llama_set_resident(struct charsiu_gpu_llama *m, int on)
{
	if (!m)
		return -1;
	if (on && !m->dec && !(m->dec = make_decoder(m)))
		return -1;
	m->resident = on != 0;
	return 0;
}

/* quantise x once, then every projection of it as one group call (or one at
 * a time under CHARSIU_GPU_NOGROUP, the control) */
static int project(struct charsiu_gpu_llama *m, const float *x, uint32_t k, const int *ids,
		   float **ys, unsigned n)
{
	if (m->npu_mode) {
		act_q1(m, x, (int)k);
		if (n > 1 && !m->nogroup)
			return charsiu_npu_matvec_flat(m->npu, ids, n, m->aq1, m->ad1, k, ys);
		for (unsigned i = 0; i < n; i++)
			if (charsiu_npu_matvec_flat(m->npu, &ids[i], 1, m->aq1, m->ad1, k, &ys[i]))
				return -1;
		return 0;
	}
	act_set(m, x, (int)k);
	if (n > 1 && !m->nogroup)
		return charsiu_gpu_matvec_q(m->dev, ids, n, m->aq, m->ad, k, ys);
	for (unsigned i = 0; i < n; i++)
		if (charsiu_gpu_matvec_q(m->dev, &ids[i], 1, m->aq, m->ad, k, &ys[i]))
			return -1;
	return 0;
}

API void charsiu_gpu_llama_close(struct charsiu_gpu_llama *m)
{
	if (!m)
		return;
	if (getenv("CHARSIU_STAGES") && m->stage_tok) {
		double tot = 0;

		for (int i = 0; i < T_COUNT; i++)
			tot += m->stage_ms[i];
		fprintf(stderr, "charsiu stages: %u tokens, %.3f ms a token\n", m->stage_tok,
			tot / m->stage_tok);
		for (int i = 0; i < T_COUNT; i++)
			fprintf(stderr, "  %-16s %8.3f ms a token   %5.1f%%\n", stage_name[i],
				m->stage_ms[i] / m->stage_tok, 100.0 * m->stage_ms[i] / tot);
	}
	charsiu_gpu_lend_pool(m->dev, NULL);
	charsiu_npu_lend_pool(m->npu, NULL);
	pool_free(m->pool);
	charsiu_gpu_decoder_free(m->dec);
	if (m->npu && getenv("CHARSIU_GPU_REPORT"))
		charsiu_npu_report(m->npu);
	charsiu_npu_close(m->npu);
	if (m->dev && getenv("CHARSIU_GPU_REPORT"))
		charsiu_gpu_report(m->dev);
	charsiu_gpu_close(m->dev);
	free(m->L);
	free(m->kcache); free(m->vcache);
	free(m->x); free(m->xb); free(m->xb2); free(m->hb); free(m->hb2);
	free(m->q); free(m->k); free(m->v); free(m->att); free(m->logits);
	free(m->aq); free(m->ad); free(m->rope_cs); free(m->aq1);
	gclose(&m->g);
	free(m);
}

static const struct gt *need(struct charsiu_gpu_llama *m, const char *name)
{
	const struct gt *t = gfind(&m->g, name);

	if (!t)
		fprintf(stderr, "charsiu: the file has no tensor %s\n", name);
	return t;
}

API struct charsiu_gpu_llama *charsiu_gpu_llama_open(const char *path, int n_ctx, int device)
{
	static const char *pname[P_N] = { "attn_q", "attn_k", "attn_v", "attn_output",
					   "ffn_gate", "ffn_up", "ffn_down" };
	struct charsiu_gpu_llama *m = calloc(1, sizeof(*m));
	const struct gt *t;
	char key[128];
	size_t kvn;
	uint32_t widest;

	if (!m)
		return NULL;
	if (gopen(&m->g, path) < 0) {
		free(m);
		return NULL;
	}
	if (strcmp(m->g.arch, "llama") || !m->g.have[K_EMBD] || !m->g.have[K_LAYERS] ||
	    !m->g.have[K_HEAD] || !m->g.have[K_FF]) {
		fprintf(stderr, "charsiu: %s is not a llama model this can read\n", path);
		goto fail;
	}
	m->n_embd = m->g.u[K_EMBD];
	m->n_layer = m->g.u[K_LAYERS];
	m->n_head = m->g.u[K_HEAD];
	m->n_head_kv = m->g.have[K_HEAD_KV] ? m->g.u[K_HEAD_KV] : m->n_head;
	m->n_ff = m->g.u[K_FF];
	m->hd = m->g.have[K_ROPE_DIM] ? m->g.u[K_ROPE_DIM] : m->n_embd / m->n_head;
	m->eps = m->g.have_f[F_EPS] ? m->g.f[F_EPS] : 1e-5f;
	m->base = m->g.have_f[F_BASE] ? m->g.f[F_BASE] : 10000.0f;
	m->n_vocab = (uint32_t)m->g.n_tokens;
	m->nogroup = getenv("CHARSIU_GPU_NOGROUP") != NULL;
	if (m->hd & 1 || !m->n_vocab || gfind(&m->g, "rope_freqs.weight")) {
		fprintf(stderr, "charsiu: unsupported head dim, vocabulary or rope table\n");
		goto fail;
	}
	{
		uint32_t ctx_train = m->g.have[K_CTX] ? m->g.u[K_CTX] : 2048;

		m->n_ctx = n_ctx > 0 ? n_ctx : (int)ctx_train;
		if (n_ctx <= 0 && m->n_ctx > 4096)
			m->n_ctx = 4096;
	}
	m->tok = need(m, "token_embd.weight");
	t = need(m, "output_norm.weight");
	if (!m->tok || !t || t->type != T_F32)
		goto fail;
	m->out_norm = (const float *)t->data;
	m->out = gfind(&m->g, "output.weight");
	if (!m->out)
		m->out = m->tok;       /* tied, as Llama 3.2 1B (src/llama.c:463-466) */

	widest = m->n_embd > m->n_ff ? m->n_embd : m->n_ff;
	m->dev = charsiu_gpu_open_ex(widest, m->n_vocab > widest ? m->n_vocab : widest,
				     m->n_layer * 9 + 2, device, 0, 1);
	if (!m->dev)
		goto fail;
	{
		/* CHARSIU_GPU_THREADS helpers for the CPU steps (0: none) */
		const char *e = getenv("CHARSIU_GPU_THREADS");
		long cpus = sysconf(_SC_NPROCESSORS_ONLN);
		int threads = e ? atoi(e) : (int)(cpus > 2 ? (cpus - 1 < 8 ? cpus - 1 : 8) : 0);

		m->pool = pool_new(threads);
		charsiu_gpu_lend_pool(m->dev, m->pool);
	}
	{
		const char *e = getenv("CHARSIU_NPU_QUANT");

		m->npu_mode = e && *e != '0';
	}
	if (m->npu_mode) {
		m->npu = charsiu_npu_open_ex(widest, m->n_vocab > widest ? m->n_vocab : widest,
					     m->n_layer * 9 + 2, device);
		m->aq1 = calloc((size_t)(widest + 31) / 32 * 32, 1);
		if (!m->npu || !m->aq1)
			goto fail;
		charsiu_npu_lend_pool(m->npu, m->pool);
	}
	m->L = calloc(m->n_layer, sizeof(*m->L));
	if (!m->L)
		goto fail;
	for (uint32_t l = 0; l < m->n_layer; l++) {
		struct layer *L = &m->L[l];

		snprintf(key, sizeof(key), "blk.%u.attn_norm.weight", l);
		if (!(t = need(m, key)) || t->type != T_F32)
			goto fail;
		L->attn_norm = (const float *)t->data;
		snprintf(key, sizeof(key), "blk.%u.ffn_norm.weight", l);
		if (!(t = need(m, key)) || t->type != T_F32)
			goto fail;
		L->ffn_norm = (const float *)t->data;
		for (int p = 0; p < P_N; p++) {
			snprintf(key, sizeof(key), "blk.%u.%s.weight", l, pname[p]);
			if (!(L->w[p] = need(m, key)))
				goto fail;
			L->id[p] = m->npu_mode
				? add_npu(m, L->w[p])
				: charsiu_gpu_add_blocks(m->dev, L->w[p]->type, L->w[p]->ne[0],
							 L->w[p]->ne[1], L->w[p]->data, key);
			if (L->id[p] < 0)
				goto fail;
		}
	}
	m->out_id = m->npu_mode ? add_npu(m, m->out)
				: charsiu_gpu_add_blocks(m->dev, m->out->type, m->out->ne[0],
							 m->out->ne[1], m->out->data, m->out->name);
	if (m->out_id < 0)
		goto fail;

	kvn = (size_t)m->n_layer * (size_t)m->n_ctx * m->n_head_kv * m->hd;
	m->kcache = calloc(kvn, sizeof(float));
	m->vcache = calloc(kvn, sizeof(float));
	m->x = calloc(m->n_embd, sizeof(float));
	m->xb = calloc(m->n_embd, sizeof(float));
	m->xb2 = calloc(m->n_embd, sizeof(float));
	m->hb = calloc(m->n_ff, sizeof(float));
	m->hb2 = calloc(m->n_ff, sizeof(float));
	m->q = calloc((size_t)m->n_head * m->hd, sizeof(float));
	m->k = calloc((size_t)m->n_head_kv * m->hd, sizeof(float));
	m->v = calloc((size_t)m->n_head_kv * m->hd, sizeof(float));
	m->att = calloc((size_t)m->n_head * m->n_ctx, sizeof(float));
	m->logits = calloc(m->n_vocab, sizeof(float));
	m->aq = calloc((size_t)(widest + 31) / 32 * 32, 1);
	m->ad = calloc((size_t)(widest + 31) / 32, sizeof(float));
	m->rope_cs = calloc(m->hd, sizeof(float));
	if (!m->rope_cs || !m->kcache || !m->vcache || !m->x || !m->xb || !m->xb2 || !m->hb || !m->hb2 ||
	    !m->q || !m->k || !m->v || !m->att || !m->logits || !m->aq || !m->ad)
		goto fail;
	{
		const char *e = getenv("CHARSIU_GPU_RESIDENT");

		if (e && atoi(e) && charsiu_gpu_llama_set_resident(m, 1))
			goto fail;
	}
	return m;
fail:
	charsiu_gpu_llama_close(m);
	return NULL;
}

static double now_ms(void)
{
	struct timespec t;

	clock_gettime(CLOCK_MONOTONIC, &t);
	return (double)t.tv_sec * 1e3 + (double)t.tv_nsec / 1e6;
}

/* One attention head of layer l at pos (src/llama.c:792-817): the scores,
 * softmax and weighted sum of this head only, so the heads can run on any
 * threads in any order with the same results. */
struct attn_job {
	struct charsiu_gpu_llama *m;
	uint32_t l;
	int pos;
	float scale;
};

static void attn_head(void *arg, int item)
{
	const struct attn_job *j = arg;
	struct charsiu_gpu_llama *m = j->m;
	uint32_t h = (uint32_t)item, l = j->l, hd = m->hd;
	uint32_t kvdim = m->n_head_kv * hd, gqa = m->n_head / m->n_head_kv;
	int pos = j->pos;
	float scale = j->scale;
	const float *qh = m->q + h * hd;
	float *att = m->att + (size_t)h * m->n_ctx;
	uint32_t kvh = h / gqa;
	float *out = m->xb + h * hd;

	/* four positions at a time: four independent chains, each summed over
	 * i in order, as src/llama.c:798-806 sums one */
	int t = 0;

	for (; t + 3 <= pos; t += 4) {
		const float *k0 = m->kcache + ((size_t)l * m->n_ctx + t) * kvdim + kvh * hd;
		const float *k1 = k0 + kvdim, *k2 = k1 + kvdim, *k3 = k2 + kvdim;
		float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;

		for (uint32_t i = 0; i < hd; i++) {
			a0 += qh[i] * k0[i];
			a1 += qh[i] * k1[i];
			a2 += qh[i] * k2[i];
			a3 += qh[i] * k3[i];
		}
		att[t] = a0 * scale;
		att[t + 1] = a1 * scale;
		att[t + 2] = a2 * scale;
		att[t + 3] = a3 * scale;
	}
	for (; t <= pos; t++) {
		const float *kt = m->kcache + ((size_t)l * m->n_ctx + t) * kvdim + kvh * hd;
		float a = 0.0f;

		for (uint32_t i = 0; i < hd; i++)
			a += qh[i] * kt[i];
		att[t] = a * scale;
	}
	softmax(att, pos + 1);
	memset(out, 0, hd * sizeof(float));
	for (t = 0; t <= pos; t++) {
		const float *vt = m->vcache + ((size_t)l * m->n_ctx + t) * kvdim + kvh * hd;
		float a = att[t];

		for (uint32_t i = 0; i < hd; i++)
			out[i] += a * vt[i];
	}
}

/* SiLU(gate) * up over one chunk of the FFN (src/llama.c:831-836) */
#define SILU_CHUNK 512

static void silu_chunk(void *arg, int item)
{
	struct charsiu_gpu_llama *m = arg;
	uint32_t i0 = (uint32_t)item * SILU_CHUNK;
	uint32_t i1 = i0 + SILU_CHUNK < m->n_ff ? i0 + SILU_CHUNK : m->n_ff;

	for (uint32_t i = i0; i < i1; i++) {
		float g = m->hb[i];

		g *= 1.0f / (1.0f + expf(-g));
		m->hb[i] = g * m->hb2[i];
	}
}

API const float *charsiu_gpu_llama_forward(struct charsiu_gpu_llama *m, int32_t token, int pos)
{
	uint32_t hd = m->hd, kvdim = m->n_head_kv * hd;
	float scale = 1.0f / sqrtf((float)hd);
	double t0 = now_ms(), t1;

#define STAGE(i) do { t1 = now_ms(); m->stage_ms[i] += t1 - t0; t0 = t1; } while (0)

	if (pos < 0 || pos >= m->n_ctx || token < 0 || (uint32_t)token >= m->tok->ne[1])
		return NULL;
	if (m->resident) {
		if (charsiu_gpu_decoder_step(m->dec, token, pos, 1, NULL))
			return NULL;
		return charsiu_gpu_decoder_logits(m->dec);
	}
	if (row_f32(m->tok, (uint64_t)token, m->x))
		return NULL;
	rope_angles(m->rope_cs, hd, pos, m->base);
	STAGE(T_EMBED);

	for (uint32_t l = 0; l < m->n_layer; l++) {
		const struct layer *L = &m->L[l];
		float *kc = m->kcache + ((size_t)l * m->n_ctx + pos) * kvdim;
		float *vc = m->vcache + ((size_t)l * m->n_ctx + pos) * kvdim;

		rmsnorm(m->xb, m->x, L->attn_norm, m->n_embd, m->eps);
		STAGE(T_ATTN_NORM);
		{
			int ids[3] = { L->id[P_Q], L->id[P_K], L->id[P_V] };
			float *ys[3] = { m->q, m->k, m->v };

			if (project(m, m->xb, m->n_embd, ids, ys, 3))
				return NULL;
		}
		STAGE(T_QKV);
		rope(m->q, m->n_head, hd, m->rope_cs);
		rope(m->k, m->n_head_kv, hd, m->rope_cs);
		memcpy(kc, m->k, kvdim * sizeof(float));
		memcpy(vc, m->v, kvdim * sizeof(float));
		STAGE(T_ROTARY);

		{
			struct attn_job job = { m, l, pos, scale };

			pool_run(m->pool, attn_head, &job, (int)m->n_head);
		}
		STAGE(T_HEADS);
		{
			int id = L->id[P_O];
			float *ys[1] = { m->xb2 };

			if (project(m, m->xb, m->n_embd, &id, ys, 1))
				return NULL;
		}
		STAGE(T_OUT_PROJ);
		for (uint32_t i = 0; i < m->n_embd; i++)
			m->x[i] += m->xb2[i];
		STAGE(T_ADD_ATTN);

		rmsnorm(m->xb, m->x, L->ffn_norm, m->n_embd, m->eps);
		STAGE(T_FFN_NORM);
		{
			int ids[2] = { L->id[P_GATE], L->id[P_UP] };
			float *ys[2] = { m->hb, m->hb2 };

			if (project(m, m->xb, m->n_embd, ids, ys, 2))
				return NULL;
		}
		STAGE(T_GATE_UP);
		pool_run(m->pool, silu_chunk, m, (int)((m->n_ff + SILU_CHUNK - 1) / SILU_CHUNK));
		STAGE(T_SWIGLU);
		{
			int id = L->id[P_DOWN];
			float *ys[1] = { m->xb2 };

			if (project(m, m->hb, m->n_ff, &id, ys, 1))
				return NULL;
		}
		STAGE(T_DOWN);
		for (uint32_t i = 0; i < m->n_embd; i++)
			m->x[i] += m->xb2[i];
		STAGE(T_ADD_FFN);
	}
	rmsnorm(m->xb, m->x, m->out_norm, m->n_embd, m->eps);
	STAGE(T_OUT_NORM);
	{
		float *ys[1] = { m->logits };

		if (project(m, m->xb, m->n_embd, &m->out_id, ys, 1))
			return NULL;
	}
	STAGE(T_VOCAB);
#undef STAGE
	m->stage_tok++;
	return m->logits;
}

/* llama_stages_report / reset (src/llama.c:719-739) */
API int charsiu_gpu_llama_stages(struct charsiu_gpu_llama *m, double *ms_per_token, int n,
				 int reset)
{
	if (!m)
		return -1;
	for (int i = 0; i < n && i < T_COUNT; i++)
		ms_per_token[i] = m->stage_tok ? m->stage_ms[i] / m->stage_tok : 0.0;
	if (reset) {
		memset(m->stage_ms, 0, sizeof(m->stage_ms));
		m->stage_tok = 0;
	}
	return T_COUNT;
}

API const char *charsiu_gpu_llama_stage_name(int i)
{
	return i >= 0 && i < T_COUNT ? stage_name[i] : "";
}

API int32_t charsiu_gpu_llama_argmax(const float *logits, uint32_t n)
{
	int32_t best = 0;

	for (uint32_t i = 1; i < n; i++)
		if (logits[i] > logits[best])
			best = (int32_t)i;
	return best;
}

/* charsiu_gpu_llama_greedy on the resident step: the argmax comes back with
 * each step, the logits only when the caller keeps them */
static int greedy_resident(struct charsiu_gpu_llama *m, const int32_t *prompt, int n_prompt,
			   int n_gen, int32_t *out, float *logits, double *gen_ms)
{
	int pos = 0;
	int32_t next = 0;
	double t0;

	for (int i = 0; i < n_prompt; i++)
		if (charsiu_gpu_decoder_step(m->dec, prompt[i], pos++,
					     logits && i == n_prompt - 1, &next))
			return -1;
	t0 = now_ms();
	for (int i = 0; i < n_gen; i++) {
		out[i] = next;
		if (logits)
			memcpy(logits + (size_t)i * m->n_vocab, charsiu_gpu_decoder_logits(m->dec),
			       (size_t)m->n_vocab * sizeof(float));
		/* as charsiu_run: every generated token is fed back */
		if (charsiu_gpu_decoder_step(m->dec, out[i], pos++, logits && i + 1 < n_gen, &next))
			return -1;
	}
	if (gen_ms)
		*gen_ms = now_ms() - t0;
	return n_gen;
}

API int charsiu_gpu_llama_greedy(struct charsiu_gpu_llama *m, const int32_t *prompt,
				 int n_prompt, int n_gen, int32_t *out, float *logits,
				 double *gen_ms)
{
	const float *lg = NULL;
	int pos = 0;
	double t0;

	if (!m || n_prompt < 1 || n_gen < 0 || n_prompt + n_gen > m->n_ctx)
		return -1;
	if (m->resident)
		return greedy_resident(m, prompt, n_prompt, n_gen, out, logits, gen_ms);
	for (int i = 0; i < n_prompt; i++)
		if (!(lg = charsiu_gpu_llama_forward(m, prompt[i], pos++)))
			return -1;
	t0 = now_ms();
	for (int i = 0; i < n_gen; i++) {
		out[i] = charsiu_gpu_llama_argmax(lg, m->n_vocab);
		if (logits)
			memcpy(logits + (size_t)i * m->n_vocab, lg, (size_t)m->n_vocab * sizeof(float));
		/* as charsiu_run: every generated token is fed back */
		if (!(lg = charsiu_gpu_llama_forward(m, out[i], pos++)))
			return -1;
	}
	if (gen_ms)
		*gen_ms = now_ms() - t0;
	return n_gen;
}

API uint32_t charsiu_gpu_llama_vocab(const struct charsiu_gpu_llama *m)
{
	return m ? m->n_vocab : 0;
}

API struct charsiu_gpu *charsiu_gpu_llama_layer(struct charsiu_gpu_llama *m)
{
	return m ? m->dev : NULL;
}

API struct charsiu_gpu_decoder *charsiu_gpu_llama_decoder(struct charsiu_gpu_llama *m)
{
	return m ? m->dec : NULL;
}

API struct charsiu_npu *charsiu_gpu_llama_npu(struct charsiu_gpu_llama *m)
{
	return m ? m->npu : NULL;
}
