/* SPDX-License-Identifier: GPL-2.0-or-later */
#ifndef CHARSIU_GPU_H
#define CHARSIU_GPU_H

/*
 * The GPU device layer: a drop-in for charsiu's NPU device layer on NVIDIA
 * B200 (sm_100a).
 *
 * Every call below is the GPU twin of one charsiu_npu_* call (declared in the
 * reference at include/charsiu_llm.h:186-200, implemented in src/npudev.c),
 * with the same conventions:
 *
 *   - NULL / -1 on failure, never abort. A failed call leaves the caller's
 *     output undefined and the caller recomputes on the CPU, as llama.c does
 *     for the NPU (src/llama.c:269-282).
 *   - Three slow or failed calls in a row retire the layer; every call after
 *     that returns -1 (src/npudev.c:560-602). The first refusal is printed once
 *     (src/npudev.c:124-138) and the report says if nothing ran on the GPU.
 *   - Not re-entrant: one decode thread calls it, before any pool fan-out
 *     (src/llama.c:261-282).
 *
 * The NPU layer takes the NPU's own per-channel int8 format; this layer takes
 * the GGUF tensor itself and computes charsiu's GGML block arithmetic
 * (src/gguf.c:1061-1107, 1149-1171) exactly: q8_0 or q4_0 weights against the
 * q8_0 activation of charsiu_act_set, int32 block dots, and the fp32 sum of
 * (d_w * d_a) * dot in block order, so y is bit-identical to gguf_matvec.
 * Weights are repacked once, at add time, into a coalesced device layout.
 *
 * The struct types are charsiu's own (include/charsiu_llm.h:51-59, 100-119;
 * include/charsiu.h:113-119, 194-225); this header only names them. Callers
 * without those headers use the flat forms (plain pointers and sizes).
 */

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CHARSIU_GPU_API __attribute__((visibility("default")))
#else
#define CHARSIU_GPU_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

struct gguf_tensor;
struct charsiu_act;
struct charsiu_job;
struct charsiu_gpu;

/* ---- lifetime ------------------------------------------------------------ */

/* charsiu_npu_open (include/charsiu_llm.h:188-189, src/npudev.c:140-233).
 * Device 0, the whole of every tensor. max_k: a multiple of 32, at most
 * 14336. NULL: no usable GPU; stay on the CPU. */
CHARSIU_GPU_API struct charsiu_gpu *charsiu_gpu_open(unsigned max_k, unsigned max_n,
				     unsigned max_tensors);

/* The same on `device`, holding only column slab `rank` of `world` of every
 * tensor added: rows [rank*N/world, (rank+1)*N/world) rounded to whole
 * 8-row groups. No counterpart in the reference (one board, one NPU); it is
 * the N-split the vendor runtime uses across NPU cores (docs/vendor-dispatch.md:43-58). */
CHARSIU_GPU_API struct charsiu_gpu *charsiu_gpu_open_ex(unsigned max_k, unsigned max_n,
					unsigned max_tensors, int device,
					unsigned rank, unsigned world);

/* charsiu_npu_close (include/charsiu_llm.h:190). NULL-safe. */
CHARSIU_GPU_API void charsiu_gpu_close(struct charsiu_gpu *g);

/* ---- weights ------------------------------------------------------------- */

/* charsiu_npu_add (include/charsiu_llm.h:191, src/npudev.c:389-461), for the
 * GGUF tensor: q8_0 or q4_0 with ne[0] = K a multiple of 32, or q6_K (the
 * head of a llama.cpp q4_0 file) with K a multiple of 256; ne[1] = N. The host
 * tensor stays the caller's. Returns an id >= 0, or -1 (tensor stays on the
 * CPU). Adding the same tensor again returns its existing id. */
CHARSIU_GPU_API int charsiu_gpu_add(struct charsiu_gpu *g, const struct gguf_tensor *w);

/* Flat form of charsiu_gpu_add: `blocks` is N rows of GGML blocks (34 bytes
 * a 32-weight q8_0 block, 18 q4_0, 210 a 256-weight q6_K super-block), row
 * major, as in a GGUF file. */
CHARSIU_GPU_API int charsiu_gpu_add_blocks(struct charsiu_gpu *g, uint32_t type, uint64_t k,
			   uint64_t n, const void *blocks, const char *name);

/* Rows this GPU holds of tensor `id`: [*row0, *row0 + *nrows). */
CHARSIU_GPU_API int charsiu_gpu_rows(const struct charsiu_gpu *g, int id, uint64_t *row0,
		     uint64_t *nrows);

/* ---- the matvec ---------------------------------------------------------- */

/* charsiu_npu_matvec (include/charsiu_llm.h:192-193, src/npudev.c:463-607):
 * y = W x from a->q and a->d (a->quantised must be set, a->n = K). y holds
 * this GPU's rows of the output (all N on an unsharded layer). */
CHARSIU_GPU_API int charsiu_gpu_matvec(struct charsiu_gpu *g, int id,
		       const struct charsiu_act *a, float *y);

/* charsiu_npu_matvec_group (include/charsiu_llm.h:195-196,
 * src/npudev.c:621-716): up to 8 projections of one activation, one launch
 * and one fence. -1: the caller falls back to single calls. */
CHARSIU_GPU_API int charsiu_gpu_matvec_group(struct charsiu_gpu *g, const int *ids, unsigned n,
			     const struct charsiu_act *a, float **ys);

/* Flat form of the group call: q is K int8 (K/32 blocks), d K/32 fp32. */
CHARSIU_GPU_API int charsiu_gpu_matvec_q(struct charsiu_gpu *g, const int *ids, unsigned n,
			 const int8_t *q, const float *d, unsigned k,
			 float **ys);

/* Batched: m activations q[m][K], d[m][K/32] against tensor id; y[m][rows].
 * Each y[i] is bit-identical to the single matvec of activation i. No
 * counterpart in the reference, which decodes one token at a time. */
CHARSIU_GPU_API int charsiu_gpu_matvec_batch(struct charsiu_gpu *g, int id, unsigned m,
			     const int8_t *q, const float *d, unsigned k,
			     float *y);

/* ---- the int8 matmul with the NPU's output stage ------------------------- */

/* What charsiu_emit_job + charsiu_submit compute for an int8 job
 * (include/charsiu.h:194-235; arithmetic of tools/charsiu_matmul.c:41-81 and
 * the output stage of src/job.c:137-177): a u8 [m][k], w u8 [n][k] (int8
 * weights, job->mm.wdtype CHARSIU_INT8), bias i32 [n]; out i8 [m][n] row
 * major, out = clamp(max(requant, 0) + offset, -128, 127). Byte-exact
 * against cpu_reference. */
CHARSIU_GPU_API int charsiu_gpu_matmul_i8(struct charsiu_gpu *g, const struct charsiu_job *job,
			  const uint8_t *a, const uint8_t *w,
			  const int32_t *bias, int8_t *out);

/* Flat form of charsiu_gpu_matmul_i8. */
CHARSIU_GPU_API int charsiu_gpu_matmul_i8_flat(struct charsiu_gpu *g, unsigned m, unsigned k,
			       unsigned n, const uint8_t *a, const uint8_t *w,
			       const int32_t *bias, float in_scale,
			       float wt_scale, float out_scale, int in_zp,
			       int wt_zp, int out_zp, int8_t *out);

/* ---- device-resident forms ------------------------------------------------ */
/*
 * For callers that keep the activation in HBM (a decode loop on the device).
 * All pointers are device pointers; the work is queued on `stream` (a
 * cudaStream_t, NULL for the layer's own) with no host synchronisation, so a
 * caller may capture it in a CUDA graph. Return 0 when queued.
 */
CHARSIU_GPU_API int charsiu_gpu_matvec_dev(struct charsiu_gpu *g, const int *ids, unsigned n,
			   const int8_t *q, const float *d, float *const *ys,
			   void *stream);
CHARSIU_GPU_API int charsiu_gpu_matvec_batch_dev(struct charsiu_gpu *g, int id, unsigned m,
				 const int8_t *q, const float *d, float *y,
				 void *stream);
/* The batched twin of charsiu_gpu_matvec_group (include/charsiu_llm.h:194-196
 * for one activation): m activations (q [m][K] int8, d [m][K/32] fp32) against
 * n <= 8 tensors of the same K, ys[i] = [m][rows of ids[i]]. From 9
 * activations, q8_0 tensors share one packing of the activations and one
 * tensor-core launch; below, the tensors of each quant type share one CUDA-core
 * launch a chunk of 8, 4 or 2 activations. */
CHARSIU_GPU_API int charsiu_gpu_matvec_batch_group_dev(struct charsiu_gpu *g, const int *ids,
						       unsigned n, unsigned m, const int8_t *q,
						       const float *d, float *const *ys,
						       void *stream);
/* ---- the matvec fused with its all-gather ------------------------------------ */
/*
 * For a layer opened with charsiu_gpu_open_ex(..., rank, world) in each of
 * `world` processes, one a GPU, that need every rank to hold the whole y (the
 * column-split decode). No counterpart in the reference (charsiu has one
 * device).
 *
 * Buffers the peers write are allocated here (charsiu_gpu_ipc_alloc: plain
 * device memory, zeroed) and shared with a 64-byte handle
 * (charsiu_gpu_ipc_handle; exchange the bytes between processes, then
 * charsiu_gpu_ipc_open gives this process's pointer to a peer's buffer;
 * charsiu_gpu_ipc_free releases either kind).
 *
 * charsiu_gpu_matvec_gather_dev runs the matvec of this rank's slab and
 * stores each y into every rank's full output full_ys[r * n + i] (tensor
 * ids[i], rank r: the whole N floats), then adds the groups it finished to
 * word signal_idx of every rank's sync array syncs[r] (uint32). With
 * wait_mult > 0 it first waits, on this GPU, until its own word wait_idx
 * reaches (epoch + wait_adj) * wait_mult, epoch being word 0, which
 * charsiu_gpu_gather_epoch_dev adds 1 to (call it at each token's start). The
 * wait gives up after one second (the layer then retires). The launches run
 * without programmatic dependence. 0 when queued on `stream`.
 */
CHARSIU_GPU_API void *charsiu_gpu_ipc_alloc(struct charsiu_gpu *g, size_t bytes);
CHARSIU_GPU_API int charsiu_gpu_ipc_handle(struct charsiu_gpu *g, void *ptr,
					   unsigned char *handle);
CHARSIU_GPU_API void *charsiu_gpu_ipc_open(struct charsiu_gpu *g, const unsigned char *handle);
CHARSIU_GPU_API void charsiu_gpu_ipc_free(struct charsiu_gpu *g, void *ptr, int opened);
/* Copy `bytes` of device memory (this GPU's, or a peer's opened above) to the
 * host; waits for it. 0 on success. */
CHARSIU_GPU_API int charsiu_gpu_read_device(struct charsiu_gpu *g, const void *dev_ptr,
					    void *host, size_t bytes);
CHARSIU_GPU_API int charsiu_gpu_gather_epoch_dev(struct charsiu_gpu *g, uint32_t *sync_local,
						 void *stream);
/* The first nonzero code a kernel of the _dev forms wrote since the last
 * call (a bounded wait that gave up), then clears it; a nonzero code retires
 * the layer, as a host call's would. 0: none. */
CHARSIU_GPU_API int charsiu_gpu_kernel_error(struct charsiu_gpu *g);
CHARSIU_GPU_API int charsiu_gpu_matvec_gather_dev(struct charsiu_gpu *g, const int *ids,
						  unsigned n, const int8_t *q, const float *d,
						  float *const *full_ys, uint32_t *const *syncs,
						  unsigned signal_idx, unsigned wait_idx,
						  unsigned wait_mult, int wait_adj, void *stream);
/* The batched form of charsiu_gpu_matvec_gather_dev: m activations (q [m][K]
 * int8, d [m][K/32] fp32, m at least CHARSIU_GPU_QMM_MIN_M, so on the tensor
 * cores) against n <= 8 q8_0 tensors of one K. Each rank's rows go straight
 * into every rank's full output full_ys[r * n + i] ([m][N] floats) from the
 * tensor-core epilogue; the waits and the arrival words are as above, except
 * that each rank adds 1 a launch (so wait_mult is the world size). No
 * counterpart in the reference. */
CHARSIU_GPU_API int charsiu_gpu_matvec_batch_gather_dev(struct charsiu_gpu *g, const int *ids,
							unsigned n, unsigned m, const int8_t *q,
							const float *d, float *const *full_ys,
							uint32_t *const *syncs, unsigned signal_idx,
							unsigned wait_idx, unsigned wait_mult,
							int wait_adj, void *stream);

/* The batched matvec of charsiu_gpu_matvec_batch_dev, for callers that
 * cannot allocate GPU memory while they run -- a server whose own memory
 * pool already owns the GPU's free memory, or a latency-bound loop that must
 * not take cudaMalloc's implicit device synchronisation (the _dev form grows
 * a staging buffer with cudaMalloc on first use). This call allocates
 * nothing: its scratch is a fixed 1 MiB array inside the library, held on
 * every GPU that loads it until exit. q8_0 tensors only; the m activations
 * are always packed into that array first, in tiles of 16 or 32 (the _dev
 * form reads them from q and d by tensor copies where it can), and must fit
 * it (m <= 64 up to
 * K = 14336), else -1 with the reason in charsiu_gpu_error. All calls on a GPU
 * share the array, so two calls running on it at the same time race. A
 * layer's first call looks up the array's device address (on the layer's
 * GPU) and keeps it; make that call before any stream capture. Every m, from
 * 1, runs on the tensor cores here (charsiu_gpu_matvec_batch_dev takes m
 * below CHARSIU_GPU_QMM_MIN_M to the CUDA cores); both are gguf_matvec bit
 * for bit, so the results are the same. No counterpart in the reference. */
CHARSIU_GPU_API int charsiu_gpu_matvec_batch_noalloc(struct charsiu_gpu *g, int id, unsigned m,
						     const int8_t *q, const float *d, float *y,
						     void *stream);
/* charsiu_act_set (src/gguf.c:829-882) on the device, bit-exact: x fp32
 * [m][k] -> q int8 [m][k rounded up to 32], d fp32 [m][k/32]. */
CHARSIU_GPU_API int charsiu_gpu_act_quantise_dev(struct charsiu_gpu *g, const float *x,
				 unsigned m, unsigned k, int8_t *q, float *d,
				 void *stream);

/* gguf_row_f32 (src/gguf.c:1217-1256) of one row of tensor id -- the
 * embedding lookup -- from the layer's copy, bit-exact: out fp32 [K]. The row
 * index is read from device memory (*row), so a captured graph can take a new
 * token each replay; an index outside the tensor writes a nonzero code that
 * charsiu_gpu_kernel_error returns. The whole tensor must be on this GPU
 * (world 1). */
CHARSIU_GPU_API int charsiu_gpu_row_dev(struct charsiu_gpu *g, int id, const int32_t *row,
					float *out, void *stream);

/* ---- the decode step on the device ------------------------------------------ */
/*
 * llama_forward (src/llama.c:743-856) with every step on the GPU: the
 * embedding row, rmsnorm, the activation quantiser, the projections (this
 * layer's matvecs), RoPE and the KV cache, attention, SiLU, the residual adds,
 * the head and llama_argmax, replayed as one CUDA graph a token. The logits
 * are the reference's bit for bit: every sum keeps the reference's order and
 * rounding, and expf is a table of the host C library's own expf over every
 * float where it is neither 1, 0 nor inf (2.2 GB of device memory, built once
 * a process and GPU, checked against expf for every float it leaves out).
 * No counterpart in the reference, which runs these steps on the CPU.
 *
 * The model: projection ids (tensors added to g) per layer in the order q, k,
 * v, o, gate, up, down; the embedding and head ids (the same tensor when the
 * head is tied); host fp32 norm weights, copied at creation; rope_cs the
 * (cos, sin) pair i of every position, [n_ctx][head_dim], as
 * src/llama.c:364-383 computes them. Requires n_head * head_dim = n_embd,
 * head_dim a multiple of 32 and at most 256, n_embd and n_ff multiples of 32, n_embd at most
 * 8192, and a layer opened with world 1.
 */
struct charsiu_gpu_decoder;

struct charsiu_gpu_decoder_desc {
	uint32_t n_embd, n_layer, n_head, n_head_kv, n_ff, head_dim, n_vocab, n_ctx;
	float rms_eps;
	int embd_id, head_id;
	const int *proj_ids;               /* [n_layer][7] */
	const float *const *attn_norm;     /* [n_layer] -> n_embd floats */
	const float *const *ffn_norm;      /* [n_layer] -> n_embd floats */
	const float *out_norm;             /* n_embd floats */
	const float *rope_cs;              /* [n_ctx][head_dim] */
};

CHARSIU_GPU_API struct charsiu_gpu_decoder *charsiu_gpu_decoder_new(
	struct charsiu_gpu *g, const struct charsiu_gpu_decoder_desc *desc);
/* The same step in charsiu's NPU number format (CHARSIU_NPU_QUANT,
 * src/llama.c:110-312): proj_ids and head_id are tensors added to npu (the
 * charsiu_npu_* layer of include/charsiu_npu.h, on g's GPU), each fed the
 * single-scale activation of charsiu_act_set (src/gguf.c:883-910) of the
 * rmsnorm, attention and SiLU outputs, computed on the device; embd_id is
 * still a tensor of g. */
struct charsiu_npu;
CHARSIU_GPU_API struct charsiu_gpu_decoder *charsiu_gpu_decoder_new_npu(
	struct charsiu_gpu *g, struct charsiu_npu *npu, const struct charsiu_gpu_decoder_desc *desc);
CHARSIU_GPU_API void charsiu_gpu_decoder_free(struct charsiu_gpu_decoder *dec);
/* One token at pos (positions run 0, 1, 2, ... as llama_forward's callers
 * step them): *next gets llama_argmax of its logits; with want_logits the
 * logits are also copied back, readable at charsiu_gpu_decoder_logits until
 * the next step. 0 on success, -1 on failure (charsiu_gpu_error says why). */
CHARSIU_GPU_API int charsiu_gpu_decoder_step(struct charsiu_gpu_decoder *dec, int32_t token,
					     int pos, int want_logits, int32_t *next);
/* The greedy loop of tools/charsiu_run.c:295-317 with the host taken out:
 * n steps from `token` at `pos`, each step's argmax the next step's token at
 * the next position, all queued at once (the argmax never leaves the device
 * between steps); out[i] gets the argmax of step i, so out[0] is what
 * charsiu_gpu_decoder_step would return for (token, pos). pos + n must not
 * pass the context. *device_ms (if given) gets the device time of the n
 * steps, from CUDA events on the decoder's stream. 0 on success, -1 on
 * failure. No counterpart in the reference. */
CHARSIU_GPU_API int charsiu_gpu_decoder_generate(struct charsiu_gpu_decoder *dec, int32_t token,
						 int pos, unsigned n, int32_t *out,
						 float *device_ms);
CHARSIU_GPU_API const float *charsiu_gpu_decoder_logits(const struct charsiu_gpu_decoder *dec);
/* kernels one step launches */
CHARSIU_GPU_API unsigned charsiu_gpu_decoder_launches(const struct charsiu_gpu_decoder *dec);

/* ---- accounting ----------------------------------------------------------- */

/* charsiu_npu_submits (include/charsiu_llm.h:197): calls that ran. */
CHARSIU_GPU_API unsigned long charsiu_gpu_calls(const struct charsiu_gpu *g);
/* kernels this layer has launched */
CHARSIU_GPU_API unsigned long charsiu_gpu_launches(const struct charsiu_gpu *g);
/* charsiu_npu_report (include/charsiu_llm.h:198, src/npudev.c:272-295) */
CHARSIU_GPU_API void charsiu_gpu_report(const struct charsiu_gpu *g);
/* the last failure, in words ("" if none) */
CHARSIU_GPU_API const char *charsiu_gpu_error(const struct charsiu_gpu *g);
/* 1 once the layer has retired itself */
CHARSIU_GPU_API int charsiu_gpu_dead(const struct charsiu_gpu *g);

/* ---- test hooks ------------------------------------------------------------ */

/* The integer block dots of tensor id against q: dots[r][K/32], int32, for
 * this GPU's rows. Bit-exact against dotq_q8_0 / dotq_q4_0's t. */
CHARSIU_GPU_API int charsiu_gpu_block_dots(struct charsiu_gpu *g, int id, const int8_t *q,
			   int32_t *dots);

/* The decode step's ordered sum on the device: the sequential fp32 sum
 * fl(...fl(fl(0 + a[0]) + a[1]) ... + a[n-1]) (rmsnorm's sum of squares,
 * src/llama.c:321-322, and the softmax sum), in both of the step's forms:
 * out[0] by one thread, out[1] by one CTA (the form the rmsnorm uses; exact
 * for non-negative finite terms, and the one-thread sum for any others).
 * a and out (2 floats) are device pointers, n <= 8192. Queued on `stream`. */
CHARSIU_GPU_API int charsiu_gpu_ordered_sum_dev(struct charsiu_gpu *g, const float *a,
						unsigned n, float *out, void *stream);

/* Host-side fault injection (no GPU fault is ever made): from call number
 * `at` on (1-based, counting matvec/group/batch/matmul calls), `count` calls
 * fail as `kind` says: 1 = the launch reports an error, 2 = the call is slow
 * (counts as a watchdog strike), 3 = the device allocation fails (at add).
 * count 0 disarms. */
CHARSIU_GPU_API int charsiu_gpu_inject(struct charsiu_gpu *g, unsigned long at,
		       unsigned long count, int kind);

#ifdef __cplusplus
}
#endif

#endif /* CHARSIU_GPU_H */
