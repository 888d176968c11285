// SPDX-License-Identifier: GPL-2.0-or-later
// The decode step on the device: charsiu's llama_forward (reference
// src/llama.c:743-856) for one token, queued once and then replayed as one
// CUDA graph a token. The projections are the layer's own matvecs (its _dev
// entry points, on this stream); everything between them is forward.cuh.
//
// A step's only host traffic is the token and its position in (8 bytes), the
// argmax out (4 bytes) and, when asked for, the logits (n_vocab floats).
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "charsiu_gpu.h"

#include "forward.cuh"
#include "layer_internal.h"
#include "npu_internal.h"

using namespace cgpu;

namespace {

// ---- the expf table ---------------------------------------------------------
//
// expf of every float with biased exponent in [EXPTAB_E0, EXPTAB_E0 +
// EXPTAB_NE), both signs, in the order exp_exact() indexes: (sign, exponent,
// mantissa). Built with this process's C library expf -- the function the
// reference's softmax and SiLU call -- so the device reads the host's own
// values. Outside that range exp_exact() returns 1, 0 or inf; the builder
// checks those answers against expf (every float below the range; the first
// binade above it and a sample beyond, where e^x is above 2^184 or below
// 2^-184 and any expf must say inf or 0) and refuses the table if one fails.

struct ExpTable {
	float *dev = nullptr;
	int refs = 0;
};
std::mutex exptab_mu;
ExpTable exptab_of[64];

template <typename F>
void parallel_for(uint64_t items, F fn)
{
	unsigned nt = std::thread::hardware_concurrency();
	nt = nt < 1 ? 1 : nt > 64 ? 64 : nt;
	std::atomic<uint64_t> next{0};
	auto work = [&]() {
		for (uint64_t i; (i = next.fetch_add(1)) < items;)
			fn(i);
	};
	std::vector<std::thread> th;
	for (unsigned t = 1; t < nt; t++)
		th.emplace_back(work);
	work();
	for (auto &t : th)
		t.join();
}

float float_of(uint32_t bits)
{
	float f;
	memcpy(&f, &bits, 4);
	return f;
}

// "" when every float outside the table gets from expf what exp_exact() gives
std::string exptab_check()
{
	std::atomic<uint64_t> bad{0}, first{~0ull};
	// below the table: 1.0f, exhaustively (2 signs x EXPTAB_E0 binades)
	const uint64_t lo_items = 2ull * EXPTAB_E0 * 16;       // 2^19 floats an item
	parallel_for(lo_items, [&](uint64_t it) {
		const uint32_t sign = (uint32_t)(it / (EXPTAB_E0 * 16));
		const uint32_t e = (uint32_t)(it / 16 % EXPTAB_E0), part = (uint32_t)(it % 16);
		uint64_t nb = 0;
		for (uint32_t m = part << 19; m < (part + 1) << 19; m++) {
			const uint32_t b = sign << 31 | e << 23 | m;
			if (expf(float_of(b)) != 1.0f) {
				nb++;
				uint64_t f = first.load();
				while (b < f && !first.compare_exchange_weak(f, b)) {
				}
			}
		}
		bad += nb;
	});
	if (bad)
		return "expf is not 1 below the table (first at bits 0x" +
		       std::to_string((unsigned long long)first.load()) + ")";
	// above: inf for x >= 128, 0 for x <= -128; the first binade whole, then
	// every 4099th float up to the largest finite one, then the infinity
	const uint32_t e_hi = EXPTAB_E0 + EXPTAB_NE;
	for (uint32_t sign = 0; sign < 2; sign++) {
		const float want = sign ? 0.0f : float_of(0x7f800000u);
		auto ok = [&](uint32_t mag) {
			const float r = expf(float_of(sign << 31 | mag));
			return r == want && !signbit(r);
		};
		for (uint32_t mag = e_hi << 23; mag < (e_hi + 1) << 23; mag++)
			if (!ok(mag))
				return std::string("expf is not ") + (sign ? "0" : "inf") +
				       " above the table";
		for (uint32_t mag = (e_hi + 1) << 23; mag < 0x7f800000u; mag += 4099)
			if (!ok(mag))
				return std::string("expf is not ") + (sign ? "0" : "inf") +
				       " above the table";
		if (!ok(0x7f7fffffu) || !ok(0x7f800000u))
			return std::string("expf is not ") + (sign ? "0" : "inf") + " above the table";
	}
	return "";
}

// the table on `device`, built and uploaded the first time; nullptr + why
float *exptab_acquire(int device, std::string &why)
{
	std::lock_guard<std::mutex> lk(exptab_mu);
	if (device < 0 || device >= 64) {
		why = "device index out of range";
		return nullptr;
	}
	ExpTable &t = exptab_of[device];
	if (t.dev) {
		t.refs++;
		return t.dev;
	}
	why = exptab_check();
	if (!why.empty())
		return nullptr;
	float *dev = nullptr;
	if (cudaMalloc(&dev, EXPTAB_ENTRIES * sizeof(float)) != cudaSuccess) {
		why = "the expf table would not allocate";
		return nullptr;
	}
	// 8 binades (256 MB) at a time through one host buffer
	constexpr uint32_t BATCH = 8;
	std::vector<float> host((size_t)BATCH << 23);
	const uint32_t nbin = 2 * EXPTAB_NE;
	for (uint32_t b0 = 0; b0 < nbin; b0 += BATCH) {
		const uint32_t nb = std::min(BATCH, nbin - b0);
		parallel_for((uint64_t)nb * 16, [&](uint64_t it) {
			const uint32_t bi = b0 + (uint32_t)(it / 16), part = (uint32_t)(it % 16);
			const uint32_t sign = bi / EXPTAB_NE, e = EXPTAB_E0 + bi % EXPTAB_NE;
			float *out = host.data() + ((size_t)(bi - b0) << 23);
			for (uint32_t m = part << 19; m < (part + 1) << 19; m++)
				out[m] = expf(float_of(sign << 31 | e << 23 | m));
		});
		if (cudaMemcpy(dev + ((size_t)b0 << 23), host.data(), ((size_t)nb << 23) * sizeof(float),
			       cudaMemcpyHostToDevice) != cudaSuccess) {
			cudaFree(dev);
			why = "the expf table would not upload";
			return nullptr;
		}
	}
	t.dev = dev;
	t.refs = 1;
	return dev;
}

void exptab_release(int device)
{
	std::lock_guard<std::mutex> lk(exptab_mu);
	if (device < 0 || device >= 64)
		return;
	ExpTable &t = exptab_of[device];
	if (t.refs > 0 && --t.refs == 0) {
		cudaFree(t.dev);
		t.dev = nullptr;
	}
}

enum { P_Q, P_K, P_V, P_O, P_GATE, P_UP, P_DOWN, P_N };

} // namespace

struct charsiu_gpu_decoder {
	charsiu_gpu *g = nullptr;
	int device = 0;
	uint32_t n_embd = 0, n_layer = 0, n_head = 0, n_head_kv = 0, n_ff = 0, hd = 0;
	uint32_t n_vocab = 0, n_ctx = 0;
	float eps = 0, scale = 0;
	std::vector<int> ids;
	int embd_id = -1, head_id = -1;
	bool pdl = true;
	// charsiu's NPU number format: the projections and the head are this NPU
	// layer's tensors, fed single-scale activations (q1, kp bytes, and *d1)
	charsiu_npu *npu = nullptr;
	int8_t *q1 = nullptr;
	float *d1 = nullptr;
	float *vf = nullptr;          // the fp32 attention / SiLU outputs before their q1
	uint32_t kp_embd = 0, kp_ff = 0;
	cudaStream_t st = nullptr;
	float *exptab = nullptr;
	float *norm = nullptr;        // [2 n_layer + 1][n_embd]: attn, ffn per layer, then out
	float *rope = nullptr;        // [n_ctx][hd]
	float *kc = nullptr, *vc = nullptr;   // [n_layer][n_ctx][kvdim]
	float *x = nullptr, *qv = nullptr, *kv = nullptr, *vv = nullptr, *xb2 = nullptr;
	float *hb = nullptr, *hb2 = nullptr, *logits = nullptr;
	int8_t *aq = nullptr;
	float *ad = nullptr;
	int *io = nullptr;            // FWD_IO_WORDS (device)
	float *part_v = nullptr;      // the argmax's per-CTA results
	uint32_t *part_i = nullptr;
	int *h_io = nullptr;          // pinned
	float *h_logits = nullptr;    // pinned
	// [mode]: 0 a host step, 1 a host step with the logits copied back, 2 a
	// step of the device-side greedy run (no copies; the argmax becomes the
	// next token on the device)
	cudaGraphExec_t exec[3] = {nullptr, nullptr, nullptr};
	bool warm[3] = {false, false, false};
	int32_t *gen_out = nullptr;   // [n_ctx] tokens of a device-side run
	int32_t *h_gen = nullptr;     // pinned copy of them
	cudaEvent_t ev[2] = {nullptr, nullptr};
	unsigned launches = 0;        // kernels a step
};

namespace {

bool fail(charsiu_gpu_decoder *dec, const char *why)
{
	layer_whine(dec->g, why);
	return false;
}

template <typename K, typename... Args>
bool launch(charsiu_gpu_decoder *dec, K kernel, unsigned grid, unsigned block, size_t smem,
	    Args... args)
{
	cudaLaunchConfig_t cfg = {};
	cfg.gridDim = dim3(grid);
	cfg.blockDim = dim3(block);
	cfg.dynamicSmemBytes = smem;
	cfg.stream = dec->st;
	cudaLaunchAttribute attr[1];
	attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	attr[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = attr;
	cfg.numAttrs = dec->pdl ? 1 : 0;
	if (cudaLaunchKernelEx(&cfg, kernel, args...) != cudaSuccess)
		return false;
	dec->launches++;
	return true;
}

bool norm_quant(charsiu_gpu_decoder *dec, const float *add, const float *w)
{
	return launch(dec, fwd_norm_quant_kernel, 1, FWD_NORM_THREADS, fwd_norm_smem(dec->n_embd),
		      dec->x, add, w, dec->n_embd, dec->eps, dec->aq, dec->ad);
}

bool matvec(charsiu_gpu_decoder *dec, const int *ids, unsigned n, float *const *ys)
{
	const unsigned long before = charsiu_gpu_launches(dec->g);
	if (charsiu_gpu_matvec_dev(dec->g, ids, n, dec->aq, dec->ad, ys, dec->st))
		return false;
	dec->launches += (unsigned)(charsiu_gpu_launches(dec->g) - before);
	return true;
}

// NPU number format: rmsnorm with the single-scale quantiser into q1 / d1
bool norm_q1(charsiu_gpu_decoder *dec, const float *add, const float *w)
{
	return launch(dec, fwd_norm_q1_kernel, 1, FWD_NORM_THREADS, fwd_norm_smem(dec->n_embd),
		      dec->x, add, w, dec->n_embd, dec->eps, dec->kp_embd, dec->q1, dec->d1);
}

bool q1_of(charsiu_gpu_decoder *dec, const float *v, uint32_t n, uint32_t kp)
{
	return launch(dec, fwd_q1_kernel, 1, FWD_Q1_THREADS, (size_t)n * 4, v, n, kp, dec->q1,
		      dec->d1);
}

bool npu_matvec(charsiu_gpu_decoder *dec, const int *ids, unsigned n, float *const *ys)
{
	const unsigned long before = npu_layer_launches(dec->npu);
	if (npu_layer_matvec_dev_d1(dec->npu, ids, n, dec->q1, dec->d1, ys, dec->st))
		return false;
	dec->launches += (unsigned)(npu_layer_launches(dec->npu) - before);
	return true;
}

// One token in the NPU number format (src/llama.c:110-312 with
// CHARSIU_NPU_QUANT): llama_forward's steps as queue_step's, every projection
// and the head an NPU-format matvec of a single-scale activation -- after
// each rmsnorm, the attention output and SiLU's.
bool queue_step_npu(charsiu_gpu_decoder *dec, int mode)
{
	const uint32_t n = dec->n_embd, kvdim = dec->n_head_kv * dec->hd;
	const size_t layer_kv = (size_t)dec->n_ctx * kvdim;
	dec->launches = 0;
	if (mode != 2 && cudaMemcpyAsync(dec->io, dec->h_io, 2 * sizeof(int),
					 cudaMemcpyHostToDevice, dec->st) != cudaSuccess)
		return fail(dec, "the step's input copy failed");
	{
		const unsigned long before = charsiu_gpu_launches(dec->g);
		if (charsiu_gpu_row_dev(dec->g, dec->embd_id, dec->io + FWD_IO_TOKEN, dec->x, dec->st))
			return fail(dec, "the embedding lookup failed");
		dec->launches += (unsigned)(charsiu_gpu_launches(dec->g) - before);
	}
	const size_t attn_smem = fwd_attention_smem(dec->n_ctx, dec->hd);
	for (uint32_t l = 0; l < dec->n_layer; l++) {
		const int *id = dec->ids.data() + (size_t)l * P_N;
		float *kc = dec->kc + l * layer_kv, *vc = dec->vc + l * layer_kv;
		if (!norm_q1(dec, l ? dec->xb2 : nullptr, dec->norm + (size_t)(2 * l) * n))
			return fail(dec, "a launch failed (attention rmsnorm)");
		{
			float *ys[3] = {dec->qv, dec->kv, dec->vv};
			if (!npu_matvec(dec, id + P_Q, 3, ys))
				return fail(dec, "the q, k, v matvec failed");
		}
		if (!launch(dec, fwd_attention_kernel, dec->n_head, FWD_ATTN_THREADS, attn_smem,
			    (const float *)dec->qv, (const float *)dec->kv, (const float *)dec->vv,
			    (const float *)dec->rope, kc, vc, (const int *)dec->io, dec->n_head,
			    dec->n_head_kv, dec->hd, dec->n_ctx, fwd_attention_tile(dec->hd), dec->scale,
			    (const float *)dec->exptab, (int8_t *)nullptr, (float *)nullptr, dec->vf) ||
		    !q1_of(dec, dec->vf, n, dec->kp_embd))
			return fail(dec, "a launch failed (attention)");
		{
			float *ys[1] = {dec->xb2};
			if (!npu_matvec(dec, id + P_O, 1, ys))
				return fail(dec, "the output projection failed");
		}
		if (!norm_q1(dec, dec->xb2, dec->norm + (size_t)(2 * l + 1) * n))
			return fail(dec, "a launch failed (ffn rmsnorm)");
		{
			float *ys[2] = {dec->hb, dec->hb2};
			if (!npu_matvec(dec, id + P_GATE, 2, ys))
				return fail(dec, "the gate, up matvec failed");
		}
		if (!launch(dec, fwd_silu_quant_kernel, (dec->n_ff + 255) / 256, 256, 0,
			    (const float *)dec->hb, (const float *)dec->hb2, dec->n_ff,
			    (const float *)dec->exptab, (int8_t *)nullptr, (float *)nullptr, dec->vf) ||
		    !q1_of(dec, dec->vf, dec->n_ff, dec->kp_ff))
			return fail(dec, "a launch failed (silu)");
		{
			float *ys[1] = {dec->xb2};
			if (!npu_matvec(dec, id + P_DOWN, 1, ys))
				return fail(dec, "the down projection failed");
		}
	}
	if (!norm_q1(dec, dec->xb2, dec->norm + (size_t)(2 * dec->n_layer) * n))
		return fail(dec, "a launch failed (final rmsnorm)");
	{
		float *ys[1] = {dec->logits};
		if (!npu_matvec(dec, &dec->head_id, 1, ys))
			return fail(dec, "the output head failed");
	}
	if (!launch(dec, fwd_argmax_kernel, FWD_ARGMAX_CTAS, FWD_ARGMAX_THREADS, 0,
		    (const float *)dec->logits, dec->n_vocab, dec->io,
		    reinterpret_cast<uint32_t *>(dec->io + FWD_IO_TICKET), dec->part_v, dec->part_i))
		return fail(dec, "a launch failed (argmax)");
	if (mode == 2)
		return launch(dec, fwd_advance_kernel, 1, 32, 0, dec->io, dec->gen_out) ||
		       fail(dec, "a launch failed (advance)");
	if (cudaMemcpyAsync(dec->h_io + FWD_IO_NEXT, dec->io + FWD_IO_NEXT, sizeof(int),
			    cudaMemcpyDeviceToHost, dec->st) != cudaSuccess)
		return fail(dec, "the step's output copy failed");
	if (mode == 1 && cudaMemcpyAsync(dec->h_logits, dec->logits, (size_t)dec->n_vocab * 4,
					 cudaMemcpyDeviceToHost, dec->st) != cudaSuccess)
		return fail(dec, "the logits copy failed");
	return true;
}

// Queue one token's work on dec->st (eagerly or into a capture).
bool queue_step(charsiu_gpu_decoder *dec, int mode)
{
	if (dec->npu)
		return queue_step_npu(dec, mode);
	const uint32_t n = dec->n_embd, kvdim = dec->n_head_kv * dec->hd;
	const size_t layer_kv = (size_t)dec->n_ctx * kvdim;
	dec->launches = 0;
	if (mode != 2 && cudaMemcpyAsync(dec->io, dec->h_io, 2 * sizeof(int),
					 cudaMemcpyHostToDevice, dec->st) != cudaSuccess)
		return fail(dec, "the step's input copy failed");
	{
		const unsigned long before = charsiu_gpu_launches(dec->g);
		if (charsiu_gpu_row_dev(dec->g, dec->embd_id, dec->io + FWD_IO_TOKEN, dec->x, dec->st))
			return fail(dec, "the embedding lookup failed");
		dec->launches += (unsigned)(charsiu_gpu_launches(dec->g) - before);
	}
	const size_t attn_smem = fwd_attention_smem(dec->n_ctx, dec->hd);
	for (uint32_t l = 0; l < dec->n_layer; l++) {
		const int *id = dec->ids.data() + (size_t)l * P_N;
		float *kc = dec->kc + l * layer_kv, *vc = dec->vc + l * layer_kv;
		if (!norm_quant(dec, l ? dec->xb2 : nullptr, dec->norm + (size_t)(2 * l) * n))
			return fail(dec, "a launch failed (attention rmsnorm)");
		{
			float *ys[3] = {dec->qv, dec->kv, dec->vv};
			if (!matvec(dec, id + P_Q, 3, ys))
				return fail(dec, "the q, k, v matvec failed");
		}
		if (!launch(dec, fwd_attention_kernel, dec->n_head, FWD_ATTN_THREADS, attn_smem,
			    (const float *)dec->qv, (const float *)dec->kv, (const float *)dec->vv,
			    (const float *)dec->rope, kc, vc, (const int *)dec->io, dec->n_head,
			    dec->n_head_kv, dec->hd, dec->n_ctx, fwd_attention_tile(dec->hd), dec->scale,
			    (const float *)dec->exptab,
			    dec->aq, dec->ad, (float *)nullptr))
			return fail(dec, "a launch failed (attention)");
		{
			float *ys[1] = {dec->xb2};
			if (!matvec(dec, id + P_O, 1, ys))
				return fail(dec, "the output projection failed");
		}
		if (!norm_quant(dec, dec->xb2, dec->norm + (size_t)(2 * l + 1) * n))
			return fail(dec, "a launch failed (ffn rmsnorm)");
		{
			float *ys[2] = {dec->hb, dec->hb2};
			if (!matvec(dec, id + P_GATE, 2, ys))
				return fail(dec, "the gate, up matvec failed");
		}
		if (!launch(dec, fwd_silu_quant_kernel, (dec->n_ff + 255) / 256, 256, 0,
			    (const float *)dec->hb, (const float *)dec->hb2, dec->n_ff,
			    (const float *)dec->exptab, dec->aq, dec->ad, (float *)nullptr))
			return fail(dec, "a launch failed (silu)");
		{
			float *ys[1] = {dec->xb2};
			if (!matvec(dec, id + P_DOWN, 1, ys))
				return fail(dec, "the down projection failed");
		}
	}
	if (!norm_quant(dec, dec->xb2, dec->norm + (size_t)(2 * dec->n_layer) * n))
		return fail(dec, "a launch failed (final rmsnorm)");
	{
		float *ys[1] = {dec->logits};
		if (!matvec(dec, &dec->head_id, 1, ys))
			return fail(dec, "the output head failed");
	}
	if (!launch(dec, fwd_argmax_kernel, FWD_ARGMAX_CTAS, FWD_ARGMAX_THREADS, 0,
		    (const float *)dec->logits, dec->n_vocab, dec->io,
		    reinterpret_cast<uint32_t *>(dec->io + FWD_IO_TICKET), dec->part_v, dec->part_i))
		return fail(dec, "a launch failed (argmax)");
	if (mode == 2)
		return launch(dec, fwd_advance_kernel, 1, 32, 0, dec->io, dec->gen_out) ||
		       fail(dec, "a launch failed (advance)");
	if (cudaMemcpyAsync(dec->h_io + FWD_IO_NEXT, dec->io + FWD_IO_NEXT, sizeof(int),
			    cudaMemcpyDeviceToHost, dec->st) != cudaSuccess)
		return fail(dec, "the step's output copy failed");
	if (mode == 1 && cudaMemcpyAsync(dec->h_logits, dec->logits, (size_t)dec->n_vocab * 4,
					 cudaMemcpyDeviceToHost, dec->st) != cudaSuccess)
		return fail(dec, "the logits copy failed");
	return true;
}

// Queue one step of `mode` (see exec): eagerly the first time (warming every
// launch cache and attribute outside any capture), captured into a graph the
// second, replayed after that.
bool run_step(charsiu_gpu_decoder *dec, int mode)
{
	if (dec->exec[mode])
		return cudaGraphLaunch(dec->exec[mode], dec->st) == cudaSuccess;
	if (!dec->warm[mode]) {
		dec->warm[mode] = queue_step(dec, mode);
		return dec->warm[mode];
	}
	cudaGraph_t graph = nullptr;
	bool ok = cudaStreamBeginCapture(dec->st, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
	const bool queued = ok && queue_step(dec, mode);
	ok = cudaStreamEndCapture(dec->st, &graph) == cudaSuccess && queued;
	ok = ok && cudaGraphInstantiate(&dec->exec[mode], graph, 0) == cudaSuccess;
	if (graph)
		cudaGraphDestroy(graph);
	return ok && cudaGraphLaunch(dec->exec[mode], dec->st) == cudaSuccess;
}

void release(charsiu_gpu_decoder *dec)
{
	for (cudaGraphExec_t &e : dec->exec)
		if (e) {
			cudaGraphExecDestroy(e);
			e = nullptr;
		}
	for (void *p : {(void *)dec->norm, (void *)dec->rope, (void *)dec->kc, (void *)dec->vc,
			(void *)dec->x, (void *)dec->qv, (void *)dec->kv, (void *)dec->vv,
			(void *)dec->xb2, (void *)dec->hb, (void *)dec->hb2, (void *)dec->logits,
			(void *)dec->aq, (void *)dec->ad, (void *)dec->io, (void *)dec->part_v,
			(void *)dec->part_i, (void *)dec->q1, (void *)dec->d1, (void *)dec->vf,
			(void *)dec->gen_out})
		if (p)
			cudaFree(p);
	for (cudaEvent_t &e : dec->ev)
		if (e)
			cudaEventDestroy(e);
	if (dec->h_io)
		cudaFreeHost(dec->h_io);
	if (dec->h_gen)
		cudaFreeHost(dec->h_gen);
	if (dec->h_logits)
		cudaFreeHost(dec->h_logits);
	if (dec->st)
		cudaStreamDestroy(dec->st);
	if (dec->exptab)
		exptab_release(dec->device);
}

// The step of either format: npu null, the GGML formats on g; else the
// projections and the head on npu (the embedding row still from g).
charsiu_gpu_decoder *build(charsiu_gpu *g, charsiu_npu *npu,
			   const struct charsiu_gpu_decoder_desc *d)
{
	if (!g || !d || !d->proj_ids || !d->attn_norm || !d->ffn_norm || !d->out_norm ||
	    !d->rope_cs || charsiu_gpu_dead(g) || (npu && npu_layer_dead(npu)))
		return nullptr;
	if (npu && npu_layer_device(npu) != layer_device(g)) {
		layer_whine(g, "the NPU-format layer is on another GPU than the layer");
		return nullptr;
	}
	if (!layer_whole(g)) {
		layer_whine(g, "the decode step needs a layer that holds whole tensors (world 1)");
		return nullptr;
	}
	const uint32_t n = d->n_embd, hd = d->head_dim;
	if (!d->n_layer || !d->n_head || !d->n_head_kv || d->n_head % d->n_head_kv || !hd ||
	    hd % 32 || hd > (uint32_t)FWD_ATTN_THREADS || d->n_head * hd != n || n % 32 ||
	    n > FWD_NORM_MAX || !d->n_ff ||
	    d->n_ff % 32 || !d->n_vocab || !d->n_ctx ||
	    fwd_attention_smem(d->n_ctx, hd) > 227 * 1024) {
		layer_whine(g, "the decode step does not take this model's shape");
		return nullptr;
	}
	// every tensor the step reads: K and rows as the forward pass needs them
	const uint32_t kvdim = d->n_head_kv * hd;
	auto check = [&](int id, uint64_t k, uint64_t rows) {
		uint64_t tk, tr;
		uint32_t ty;
		if (npu)
			return npu_layer_tensor(npu, id, &tk, &tr, &ty) && tk == k && tr == rows;
		return layer_tensor(g, id, &tk, &tr, &ty) && tk == k && tr == rows;
	};
	for (uint32_t l = 0; l < d->n_layer; l++) {
		const int *id = d->proj_ids + (size_t)l * P_N;
		if (!check(id[P_Q], n, n) || !check(id[P_K], n, kvdim) || !check(id[P_V], n, kvdim) ||
		    !check(id[P_O], n, n) || !check(id[P_GATE], n, d->n_ff) ||
		    !check(id[P_UP], n, d->n_ff) || !check(id[P_DOWN], d->n_ff, n)) {
			layer_whine(g, "a projection's shape is not the model's");
			return nullptr;
		}
	}
	{
		uint64_t tk, tr;
		uint32_t ty;
		if (!check(d->head_id, n, d->n_vocab) || !layer_tensor(g, d->embd_id, &tk, &tr, &ty) ||
		    tk != n || tr < d->n_vocab) {
			layer_whine(g, "the head or embedding shape is not the model's");
			return nullptr;
		}
	}

	charsiu_gpu_decoder *dec = new (std::nothrow) charsiu_gpu_decoder;
	if (!dec)
		return nullptr;
	dec->g = g;
	dec->device = layer_device(g);
	dec->n_embd = n;
	dec->n_layer = d->n_layer;
	dec->n_head = d->n_head;
	dec->n_head_kv = d->n_head_kv;
	dec->n_ff = d->n_ff;
	dec->hd = hd;
	dec->n_vocab = d->n_vocab;
	dec->n_ctx = d->n_ctx;
	dec->eps = d->rms_eps;
	dec->scale = 1.0f / sqrtf((float)hd);        // src/llama.c:748
	dec->ids.assign(d->proj_ids, d->proj_ids + (size_t)d->n_layer * P_N);
	dec->embd_id = d->embd_id;
	dec->head_id = d->head_id;
	dec->pdl = !layer_no_pdl(g);
	dec->npu = npu;
	dec->kp_embd = (n + 15) / 16 * 16;
	dec->kp_ff = (d->n_ff + 15) / 16 * 16;
	cudaSetDevice(dec->device);

	std::string why;
	dec->exptab = exptab_acquire(dec->device, why);
	if (!dec->exptab) {
		layer_whine(g, why.c_str());
		release(dec);
		delete dec;
		return nullptr;
	}
	const size_t kvn = (size_t)d->n_layer * d->n_ctx * kvdim;
	const uint32_t widest = std::max(n, d->n_ff);
	bool ok = cudaStreamCreateWithFlags(&dec->st, cudaStreamNonBlocking) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->norm, (size_t)(2 * d->n_layer + 1) * n * 4) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->rope, (size_t)d->n_ctx * hd * 4) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->kc, kvn * 4) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->vc, kvn * 4) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->x, (size_t)n * 4) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->qv, (size_t)n * 4) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->kv, (size_t)kvdim * 4) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->vv, (size_t)kvdim * 4) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->xb2, (size_t)n * 4) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->hb, (size_t)d->n_ff * 4) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->hb2, (size_t)d->n_ff * 4) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->logits, (size_t)d->n_vocab * 4) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->aq, widest) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->ad, (size_t)widest / 32 * 4) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->io, FWD_IO_WORDS * sizeof(int)) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->part_v, FWD_ARGMAX_CTAS * sizeof(float)) == cudaSuccess;
	ok = ok && cudaMalloc(&dec->part_i, FWD_ARGMAX_CTAS * sizeof(uint32_t)) == cudaSuccess;
	ok = ok && cudaHostAlloc(&dec->h_io, FWD_IO_WORDS * sizeof(int), cudaHostAllocDefault) ==
			   cudaSuccess;
	ok = ok && cudaHostAlloc(&dec->h_logits, (size_t)d->n_vocab * 4, cudaHostAllocDefault) ==
			   cudaSuccess;
	ok = ok && cudaMalloc(&dec->gen_out, (size_t)d->n_ctx * sizeof(int32_t)) == cudaSuccess;
	ok = ok && cudaHostAlloc(&dec->h_gen, (size_t)d->n_ctx * sizeof(int32_t),
				 cudaHostAllocDefault) == cudaSuccess;
	ok = ok && cudaEventCreate(&dec->ev[0]) == cudaSuccess &&
	     cudaEventCreate(&dec->ev[1]) == cudaSuccess;
	if (npu) {
		ok = ok && cudaMalloc(&dec->q1, std::max(dec->kp_embd, dec->kp_ff)) == cudaSuccess;
		ok = ok && cudaMalloc(&dec->d1, sizeof(float)) == cudaSuccess;
		ok = ok && cudaMalloc(&dec->vf, (size_t)widest * 4) == cudaSuccess;
	}
	if (ok) {
		for (uint32_t l = 0; l < d->n_layer && ok; l++) {
			ok = cudaMemcpy(dec->norm + (size_t)(2 * l) * n, d->attn_norm[l], (size_t)n * 4,
					cudaMemcpyHostToDevice) == cudaSuccess;
			ok = ok && cudaMemcpy(dec->norm + (size_t)(2 * l + 1) * n, d->ffn_norm[l],
					      (size_t)n * 4, cudaMemcpyHostToDevice) == cudaSuccess;
		}
		ok = ok && cudaMemcpy(dec->norm + (size_t)(2 * d->n_layer) * n, d->out_norm,
				      (size_t)n * 4, cudaMemcpyHostToDevice) == cudaSuccess;
		ok = ok && cudaMemcpy(dec->rope, d->rope_cs, (size_t)d->n_ctx * hd * 4,
				      cudaMemcpyHostToDevice) == cudaSuccess;
		ok = ok && cudaMemset(dec->kc, 0, kvn * 4) == cudaSuccess;
		ok = ok && cudaMemset(dec->vc, 0, kvn * 4) == cudaSuccess;
		ok = ok && cudaMemset(dec->io, 0, FWD_IO_WORDS * sizeof(int)) == cudaSuccess;
	}
	if (ok && fwd_norm_smem(n) > 48 * 1024)
		ok = cudaFuncSetAttribute(npu ? (const void *)fwd_norm_q1_kernel
					      : (const void *)fwd_norm_quant_kernel,
					  cudaFuncAttributeMaxDynamicSharedMemorySize,
					  (int)fwd_norm_smem(n)) == cudaSuccess;
	if (ok && npu && (size_t)widest * 4 > 48 * 1024)
		ok = widest * 4 <= 227 * 1024 &&
		     cudaFuncSetAttribute((const void *)fwd_q1_kernel,
					  cudaFuncAttributeMaxDynamicSharedMemorySize,
					  (int)(widest * 4)) == cudaSuccess;
	const size_t attn_smem = fwd_attention_smem(d->n_ctx, hd);
	if (ok && attn_smem > 48 * 1024)
		ok = cudaFuncSetAttribute((const void *)fwd_attention_kernel,
					  cudaFuncAttributeMaxDynamicSharedMemorySize,
					  (int)attn_smem) == cudaSuccess;
	if (!ok) {
		layer_whine(g, "the decode step's buffers would not allocate");
		release(dec);
		delete dec;
		return nullptr;
	}
	memset(dec->h_io, 0, FWD_IO_WORDS * sizeof(int));
	return dec;
}

} // namespace

extern "C" {

struct charsiu_gpu_decoder *charsiu_gpu_decoder_new(struct charsiu_gpu *g,
						    const struct charsiu_gpu_decoder_desc *d)
{
	return build(g, nullptr, d);
}

struct charsiu_gpu_decoder *charsiu_gpu_decoder_new_npu(struct charsiu_gpu *g,
							struct charsiu_npu *npu,
							const struct charsiu_gpu_decoder_desc *d)
{
	return npu ? build(g, npu, d) : nullptr;
}

void charsiu_gpu_decoder_free(struct charsiu_gpu_decoder *dec)
{
	if (!dec)
		return;
	cudaSetDevice(dec->device);
	if (dec->st)
		cudaStreamSynchronize(dec->st);
	release(dec);
	delete dec;
}

int charsiu_gpu_decoder_generate(struct charsiu_gpu_decoder *dec, int32_t token, int pos,
				 unsigned n, int32_t *out, float *device_ms)
{
	if (!dec || !out || charsiu_gpu_dead(dec->g))
		return -1;
	if (pos < 0 || token < 0 || (uint32_t)token >= dec->n_vocab || !n ||
	    (uint64_t)pos + n > dec->n_ctx) {
		layer_whine(dec->g, "token or positions out of range");
		return -1;
	}
	cudaSetDevice(dec->device);
	dec->h_io[FWD_IO_TOKEN] = token;
	dec->h_io[FWD_IO_POS] = pos;
	dec->h_io[FWD_IO_STEP] = 0;
	bool ok = cudaMemcpyAsync(dec->io + FWD_IO_TOKEN, dec->h_io + FWD_IO_TOKEN, 2 * sizeof(int),
				  cudaMemcpyHostToDevice, dec->st) == cudaSuccess &&
		  cudaMemcpyAsync(dec->io + FWD_IO_STEP, dec->h_io + FWD_IO_STEP, sizeof(int),
				  cudaMemcpyHostToDevice, dec->st) == cudaSuccess &&
		  cudaEventRecord(dec->ev[0], dec->st) == cudaSuccess;
	// (the first step of a run may warm or capture the graph; the run's
	// device time still covers every step)
	for (unsigned i = 0; i < n && ok; i++)
		ok = run_step(dec, 2);
	ok = ok && cudaEventRecord(dec->ev[1], dec->st) == cudaSuccess &&
	     cudaMemcpyAsync(dec->h_gen, dec->gen_out, (size_t)n * sizeof(int32_t),
			     cudaMemcpyDeviceToHost, dec->st) == cudaSuccess;
	if (!ok) {
		layer_whine(dec->g, "the device-side greedy run would not launch");
		cudaStreamSynchronize(dec->st);
		cudaGetLastError();
		return -1;
	}
	const cudaError_t e = cudaStreamSynchronize(dec->st);
	if (e != cudaSuccess) {
		layer_whine(dec->g, cudaGetErrorString(e));
		return -1;
	}
	if (charsiu_gpu_kernel_error(dec->g))
		return -1;
	memcpy(out, dec->h_gen, (size_t)n * sizeof(int32_t));
	if (device_ms && cudaEventElapsedTime(device_ms, dec->ev[0], dec->ev[1]) != cudaSuccess)
		*device_ms = -1.0f;
	return 0;
}

int charsiu_gpu_decoder_step(struct charsiu_gpu_decoder *dec, int32_t token, int pos,
			     int want_logits, int32_t *next)
{
	if (!dec || charsiu_gpu_dead(dec->g))
		return -1;
	if (pos < 0 || (uint32_t)pos >= dec->n_ctx || token < 0 || (uint32_t)token >= dec->n_vocab) {
		layer_whine(dec->g, "token or position out of range");
		return -1;
	}
	cudaSetDevice(dec->device);
	dec->h_io[FWD_IO_TOKEN] = token;
	dec->h_io[FWD_IO_POS] = pos;
	if (!run_step(dec, want_logits ? 1 : 0)) {
		layer_whine(dec->g, "the decode step would not launch");
		cudaStreamSynchronize(dec->st);
		cudaGetLastError();
		return -1;
	}
	const cudaError_t e = cudaStreamSynchronize(dec->st);
	if (e != cudaSuccess) {
		layer_whine(dec->g, cudaGetErrorString(e));
		return -1;
	}
	if (charsiu_gpu_kernel_error(dec->g))
		return -1;
	if (next)
		*next = dec->h_io[FWD_IO_NEXT];
	return 0;
}

int charsiu_gpu_ordered_sum_dev(struct charsiu_gpu *g, const float *a, unsigned n, float *out,
				void *stream)
{
	if (!g || !a || !out || !n || n > ORDERED_SUM_MAX_N)
		return -1;
	cudaSetDevice(layer_device(g));
	ordered_sum_kernel<<<1, ORDERED_SUM_THREADS, 0, (cudaStream_t)stream>>>(a, n, out);
	return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

const float *charsiu_gpu_decoder_logits(const struct charsiu_gpu_decoder *dec)
{
	return dec ? dec->h_logits : nullptr;
}

unsigned charsiu_gpu_decoder_launches(const struct charsiu_gpu_decoder *dec)
{
	return dec ? dec->launches : 0;
}

} // extern "C"
