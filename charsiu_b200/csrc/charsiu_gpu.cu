// SPDX-License-Identifier: GPL-2.0-or-later
// The GPU device layer: the host side of include/charsiu_gpu.h.
//
// It plays the part src/npudev.c plays for the NPU: it owns the device, the
// repacked weights and the staging buffers, turns one projection (or a group
// of projections of one activation) into one kernel launch, waits with a
// deadline, keeps the time split, retires itself after three slow or failed
// calls, and says so.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>          // PFN_cuTensorMapEncodeTiled

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <new>
#include <string>
#include <vector>

#include "charsiu_gpu.h"

#include "aux_kernels.cuh"
#include "i8mm_tc.cuh"
#include "qmv.cuh"
#include "qmv1.cuh"
#include "qmvm.cuh"
#include "q6k.cuh"
#include "qmm_tc.cuh"
#include "ref_abi.h"

#include "host_copy.h"
#include <unistd.h>

using namespace cgpu;

namespace {

constexpr unsigned MAX_K = 14336;

double now_us()
{
	timespec t;
	clock_gettime(CLOCK_MONOTONIC, &t);
	return (double)t.tv_sec * 1e6 + (double)t.tv_nsec / 1e3;
}

unsigned env_u(const char *name, unsigned dflt)
{
	const char *e = getenv(name);
	return e ? (unsigned)strtoul(e, nullptr, 0) : dflt;
}

struct Ent {
	const void *key;          // the caller's gguf_tensor, for re-adds
	char name[80];
	uint32_t type, nb;
	uint64_t k, n;            // the whole tensor
	uint64_t row0, rows;      // this GPU's slab
	uint32_t groups;
	uint8_t *data;
	size_t bytes;
	double weight_mb;         // of this GPU's slab
};

template <typename T>
bool grow_dev(T *&p, size_t &cap, size_t want)
{
	if (want <= cap)
		return true;
	if (p)
		cudaFree(p);
	p = nullptr;
	cap = 0;
	if (cudaMalloc(&p, want * sizeof(T)) != cudaSuccess)
		return false;
	cap = want;
	return true;
}

// Pinned host memory, mapped into the device's address space (the direct
// host call's kernels read and write it in place).
template <typename T>
bool grow_host(T *&p, size_t &cap, size_t want)
{
	if (want <= cap)
		return true;
	if (p)
		cudaFreeHost(p);
	p = nullptr;
	cap = 0;
	if (cudaHostAlloc(&p, want * sizeof(T), cudaHostAllocMapped) != cudaSuccess)
		return false;
	cap = want;
	return true;
}

// The device address of mapped host memory.
template <typename T>
T *dev_view(T *host)
{
	void *d = nullptr;
	if (cudaHostGetDevicePointer(&d, (void *)host, 0) != cudaSuccess)
		return nullptr;
	return static_cast<T *>(d);
}

// One host call captured as a CUDA graph: tensors ids[0..n) at K = k.
struct CallGraph {
	int ids[8];
	unsigned n, k;
	cudaGraphExec_t exec;
};

} // namespace

struct charsiu_gpu {
	int device = 0;
	unsigned rank = 0, world = 1, max_k = 0, max_n = 0, max_tensors = 0;
	int sm_count = 0;
	cudaStream_t stream = nullptr;
	cudaEvent_t ev_k0 = nullptr, ev_k1 = nullptr, ev_done = nullptr;
	std::vector<Ent> ent;

	// host-call staging: the activation as one [q | d] block, and every y
	uint8_t *d_act = nullptr, *h_act = nullptr;
	float *d_y = nullptr, *h_y = nullptr;
	size_t cap_dact = 0, cap_hact = 0, cap_dy = 0, cap_hy = 0;
	int8_t *d_q = nullptr;              // block-dot test hook
	size_t cap_dq = 0;
	uint8_t *d_pack = nullptr;          // packed activation tiles of the batched path
	size_t cap_pack = 0;
	std::vector<CallGraph> graphs;
	uint8_t *d_i8 = nullptr, *h_i8 = nullptr;
	size_t cap_di8 = 0, cap_hi8 = 0;
	int32_t *d_dots = nullptr;
	size_t cap_dots = 0;
	// a kernel whose wait gave up writes here: mapped host memory, read after
	// the call's event without another copy
	volatile int *h_err = nullptr;
	int *d_err = nullptr;
	// direct host calls: [0] CTAs done (device), [2..3] start stamp; the flag
	// words the last CTA raises (mapped host memory), and their sequence
	uint32_t *d_sync = nullptr;
	uint32_t *d_gather_count = nullptr;   // the fused gather's CTAs-done count
	volatile uint32_t *h_flag = nullptr;
	uint32_t *d_flag = nullptr;
	uint32_t seq = 0;
	QmvInline<QMV_INLINE_MAX_WORDS> *inl = nullptr;    // the direct call's kernel arguments
	I8Inline<I8_INLINE_W2> *i8inl = nullptr;            // and the int8 direct call's
	// host threads for large copies: the layer's own, or lent by the decode
	// loop that owns this layer (one set of threads serving both)
	struct pool *copy_pool = nullptr;
	bool copy_pool_tried = false, copy_pool_owned = false;
	bool direct = true;  // CHARSIU_GPU_DIRECT=0: every host call through a graph with copies
	bool smem_set[64] = {};
	uint8_t *noalloc_scratch = nullptr;  // the allocation-free call's array, on this device
	// CTAs per SM for (m, nb): asked of the driver once, never during capture
	std::vector<std::pair<uint64_t, int>> occ;

	unsigned long calls = 0, launches = 0, call_no = 0;
	double busy_us = 0, h2d_us = 0, kern_ms = 0, d2h_us = 0, weight_mb = 0;
	double slow_us = 100000;
	int strikes = 0, dead = 0, whined = 0;
	int no_pdl = 0;     // CHARSIU_GPU_NO_PDL: launch without programmatic dependence (control)
	// CHARSIU_GPU_PDL_EARLY (default 1): the M = 1 matvec lets its successor
	// start once all its CTAs have started, not once they have staged the
	// activation (1B decode step 0.653 -> 0.626 ms, token chain 0.302 -> 0.295)
	int pdl_early = 1;
	// CHARSIU_GPU_GATHER_PDL (default 1): the fused matvec + gather launches
	// with programmatic dependence too. Its CTAs then start while the launch
	// before is still running on this GPU and load their first weights; each
	// waits for that launch to finish (griddepcontrol.wait) before it waits
	// on the other ranks' arrivals, so it never waits on a kernel of its own
	// GPU that might not be running.
	int gather_pdl = 1;
	uint32_t qmm_na = 0;   // CHARSIU_GPU_QMM_NA: activations a tensor-core tile (16, 32; 0 = by m)
	bool qmm_pre = false;  // CHARSIU_GPU_QMM_PRE=1: the MMA adds the float-bias constant (slower)
	// CHARSIU_GPU_QMM_MIN_M: q8_0 batches of fewer activations run on the CUDA
	// cores (qmvm_kernel). Measured crossover on the 1B decode step: the CUDA
	// cores win at 2, 4 and 8 activations (0.46 / 0.62 / 1.01 ms against
	// 1.27 / 1.28 / 1.28), the tensor cores from 16 (1.29 against 1.96 ms).
	uint32_t qmm_min_m = 9;
	unsigned long inj_at = 0, inj_count = 0;
	int inj_kind = 0;
	std::string err;
};

namespace {

void drop_graphs(charsiu_gpu *g)
{
	for (CallGraph &c : g->graphs)
		if (c.exec)
			cudaGraphExecDestroy(c.exec);
	g->graphs.clear();
}

// Say why, once (the reference's whine(), src/npudev.c:124-138): a silent
// fallback to the CPU produces results that look like GPU evidence.
void whine(charsiu_gpu *g, const char *fmt, ...)
{
	char buf[256];
	va_list ap;
	va_start(ap, fmt);
	vsnprintf(buf, sizeof(buf), fmt, ap);
	va_end(ap);
	g->err = buf;
	if (g->whined)
		return;
	g->whined = 1;
	fprintf(stderr, "charsiu: NOT on the GPU -- %s\n", buf);
}

bool injected(charsiu_gpu *g, int kind)
{
	return g->inj_kind == kind && g->inj_count && g->call_no >= g->inj_at &&
	       g->call_no < g->inj_at + g->inj_count;
}

void retire(charsiu_gpu *g, const char *why)
{
	if (g->dead)
		return;
	g->dead = 1;
	g->strikes = 3;
	fprintf(stderr, "charsiu: the GPU path is retired (%s); everything from here "
			"runs on the CPU\n", why);
}

// Wait for ev_done with the reference's budget: CHARSIU_GPU_SLOW_US plus a
// millisecond a megabyte (src/npudev.c:560-573). Slow counts a strike, three
// in a row retire the layer. A call that has not finished 10 s past its
// budget retires it at once; its buffers are then never touched again.
int finish(charsiu_gpu *g, double t0, double mb, unsigned k, unsigned n)
{
	const double budget = g->slow_us + mb * 1000.0;
	cudaError_t e;

	while ((e = cudaEventQuery(g->ev_done)) == cudaErrorNotReady) {
		if (now_us() - t0 > budget + 10e6) {
			whine(g, "a call did not finish (K=%u N=%u)", k, n);
			retire(g, "it stopped answering");
			return -1;
		}
	}
	if (e != cudaSuccess) {
		whine(g, "CUDA error %s (K=%u N=%u)", cudaGetErrorString(e), k, n);
		retire(g, "a CUDA error");
		return -1;
	}
	if (*g->h_err) {
		*g->h_err = 0;
		whine(g, "a kernel wait gave up (K=%u N=%u)", k, n);
		retire(g, "a kernel wait gave up");
		return -1;
	}
	double took = now_us() - t0;
	if (injected(g, 2))
		took = budget + 1.0;
	if (took > budget) {
		if (++g->strikes >= 3) {
			whine(g, "three slow calls in a row (K=%u N=%u)", k, n);
			retire(g, "it stopped answering in time");
			return -1;
		}
	} else {
		g->strikes = 0;
	}
	return 0;
}

// Fill QmvParams for tensors ids[0..n) with outputs at ys[i] (device).
void fill_params(charsiu_gpu *g, QmvParams &p, const int *ids, unsigned n, float *const *ys,
		 uint32_t k, const int8_t *q, const float *d)
{
	memset(&p, 0, sizeof(p));
	uint32_t acc = 0;
	for (unsigned i = 0; i < n; i++) {
		const Ent &e = g->ent[ids[i]];
		QmvTensor &t = p.t[i];
		t.data = e.data;
		t.y = ys[i];
		t.type = e.type;
		t.rows = (uint32_t)e.rows;
		t.groups = e.groups;
		acc += e.groups;
		t.group_end = acc;
		t.y_stride = (uint32_t)e.rows;
	}
	p.ntensor = n;
	p.total_groups = acc;
	p.k = k;
	p.nb = k / 32;
	p.q = q;
	p.d = d;
	p.err = g->d_err;
}

// M = 1 runs qmv1_kernel<W, Q8, TWO> (W warps share one 8-row group, one or
// two segments a warp; every tensor of the launch has the same quant type);
// M = 2, 4, 8 run qmvm_kernel<W, Q8, TWO, M> (the same shapes). Both sum blocks in the
// reference's order.
//
// `inl` (M = 1 only): a QmvInline<QMV_INLINE_MAX_WORDS> whose .p is p and
// whose words hold the activation; the launch then runs qmv1_inline_kernel,
// which reads the activation from its parameters (the first
// QmvInline<AW> bytes of the buffer, AW by the shape).
//
// `gth` (M = 1 only): the launch is qmv1_gather_kernel, the matvec fused with
// its all-gather over peer memory; it goes without programmatic dependence,
// so its wait for the other ranks never overlaps a kernel of its own GPU.
int launch_qmv(charsiu_gpu *g, int m, const QmvParams &p, cudaStream_t st,
	       const void *inl = nullptr, const QmvGather *gth = nullptr)
{
	static const void *const qmv1_gather_fns[4][2] = {
		{(const void *)qmv1_gather_kernel<4, false, false>,
		 (const void *)qmv1_gather_kernel<4, true, false>},
		{(const void *)qmv1_gather_kernel<8, false, false>,
		 (const void *)qmv1_gather_kernel<8, true, false>},
		{(const void *)qmv1_gather_kernel<8, false, true>,
		 (const void *)qmv1_gather_kernel<8, true, true>},
		{(const void *)qmv1_gather_kernel<16, false, true>,
		 (const void *)qmv1_gather_kernel<16, true, true>},
	};
	static const void *const qmv1_fns[4][2] = {
		{(const void *)qmv1_kernel<4, false, false>, (const void *)qmv1_kernel<4, true, false>},
		{(const void *)qmv1_kernel<8, false, false>, (const void *)qmv1_kernel<8, true, false>},
		{(const void *)qmv1_kernel<8, false, true>, (const void *)qmv1_kernel<8, true, true>},
		{(const void *)qmv1_kernel<16, false, true>, (const void *)qmv1_kernel<16, true, true>},
	};
	static const void *const qmv1_inline_fns[4][2] = {
		{(const void *)qmv1_inline_kernel<4, false, false, 144>,
		 (const void *)qmv1_inline_kernel<4, true, false, 144>},
		{(const void *)qmv1_inline_kernel<8, false, false, 576>,
		 (const void *)qmv1_inline_kernel<8, true, false, 576>},
		{(const void *)qmv1_inline_kernel<8, false, true, 576>,
		 (const void *)qmv1_inline_kernel<8, true, true, 576>},
		{(const void *)qmv1_inline_kernel<16, false, true, 1008>,
		 (const void *)qmv1_inline_kernel<16, true, true, 1008>},
	};
	static const int qmv1_warps[4] = {4, 8, 8, 16};
	const void *fn = nullptr;
	size_t smem = 0;
	int threads = 0, slot = 0;
	const bool q8 = p.t[0].type == TYPE_Q8_0;
	const uint32_t nseg = nsegments(p.nb);
	// (M >= 4 with 9..16 segments takes the 16-warp shape, one segment a
	// warp: its term buffers hold the CTA to one an SM, and the extra warps
	// cover more latency -- the 1B decode step at M = 4 / 8: 0.506 -> 0.463,
	// 0.797 -> 0.746 ms; at M = 2, with room for more CTAs, it lost 6 %)
	const int shape = nseg <= 4 ? 0 : nseg <= 8 ? 1 : (nseg <= 16 && m < 4) ? 2 : 3;

	if (m == 1) {
		threads = qmv1_warps[shape] * 32;
		smem = qmv1_smem_bytes(p.nb);
		// 10..17, inline 24..31, gather 56..63; q6_K 4..7, the tensor cores 19..23, M > 1 32..55
		slot = (gth ? 56 : inl ? 24 : 10) + 2 * shape + (q8 ? 1 : 0);
		fn = (gth ? qmv1_gather_fns : inl ? qmv1_inline_fns : qmv1_fns)[shape][q8 ? 1 : 0];
	} else if (inl || gth) {
		return -1;
	} else {
		// M = 2, 4, 8: qmvm_kernel, the same shapes as M = 1
#define QMVM_ROW(W, TWO, M) \
	{(const void *)qmvm_kernel<W, false, TWO, M>, (const void *)qmvm_kernel<W, true, TWO, M>}
		static const void *const qmvm_fns[4][3][2] = {
			{QMVM_ROW(4, false, 2), QMVM_ROW(4, false, 4), QMVM_ROW(4, false, 8)},
			{QMVM_ROW(8, false, 2), QMVM_ROW(8, false, 4), QMVM_ROW(8, false, 8)},
			{QMVM_ROW(8, true, 2), QMVM_ROW(8, true, 4), QMVM_ROW(8, true, 8)},
			{QMVM_ROW(16, true, 2), QMVM_ROW(16, true, 4), QMVM_ROW(16, true, 8)},
		};
#undef QMVM_ROW
		const int mi = m == 2 ? 0 : m == 4 ? 1 : m == 8 ? 2 : -1;
		if (mi < 0)
			return -1;
		threads = qmv1_warps[shape] * 32;
		smem = qmvm_smem_bytes(m, p.nb);
		if (smem > QMV_SMEM_MAX)
			return -1;
		slot = 32 + (2 * shape + (q8 ? 1 : 0)) * 3 + mi;    // 32..55
		fn = qmvm_fns[shape][mi][q8 ? 1 : 0];
	}
	if (!g->smem_set[slot]) {
		if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
					 (int)QMV_SMEM_MAX) != cudaSuccess)
			return -1;
		g->smem_set[slot] = true;
	}
	const uint64_t key = (uint64_t)slot << 32 | p.nb;
	int occ = 0;
	for (const auto &kv : g->occ)
		if (kv.first == key)
			occ = kv.second;
	if (!occ) {
		if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, threads, smem) !=
			    cudaSuccess || occ < 1)
			return -1;
		g->occ.emplace_back(key, occ);
	}
	unsigned grid = (unsigned)occ * g->sm_count;
	if (p.total_groups < grid)
		grid = p.total_groups ? p.total_groups : 1;

	cudaLaunchConfig_t cfg = {};
	cfg.gridDim = dim3(grid);
	cfg.blockDim = dim3(threads);
	cfg.dynamicSmemBytes = smem;
	cfg.stream = st;
	cudaLaunchAttribute attr[1];
	attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	attr[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = attr;
	cfg.numAttrs = g->no_pdl || (gth && !g->gather_pdl) ? 0 : 1;
	QmvParams arg = p;
	arg.early_trigger = g->pdl_early && (!gth || g->gather_pdl) ? 1u : 0u;
	if (inl)
		reinterpret_cast<QmvParams *>(const_cast<void *>(inl))->early_trigger =
			arg.early_trigger;
	QmvGather garg = gth ? *gth : QmvGather{};
	void *args[2] = {inl ? const_cast<void *>(inl) : (void *)&arg, &garg};
	const cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
	if (e != cudaSuccess)
		return -1;
	g->launches++;
	return 0;
}

// The batched q8_0 path on the tensor cores: pack the m activations into MMA
// tiles of NA (16 or 32) rows once, then one persistent launch over every
// (128-row tile, NA activations) unit of the tensors `ids` (same K, at most
// QMM_MAX_TENSORS). NA = 16 for m <= 16, else 32 (CHARSIU_GPU_QMM_NA picks
// one for every m). `pack` (device) holds at least qmm_pack_bytes(qmm_na(g, m),
// m, nb), which covers every NA a launch may pick (qmm_launch_na).
uint32_t qmm_na(const charsiu_gpu *g, uint32_t m)
{
	if (g->qmm_na)
		return g->qmm_na;
	return m <= 16 ? 16 : 32;
}

// The (NA, EC) of one launch of `tiles` row tiles: the smallest units that
// still run in one round on the SMs. An epilogue warp's share of a unit is
// the same in every shape (32 rows, 8 activations; 4 in the 4-wide units), so
// a smaller unit takes no longer than a larger one and more of them run side
// by side; once they
// no longer fit one round, the larger units' fewer rounds win. At m = 64 the
// 2048-row launches (o, down) run 128 units of (tile, 8 activations) instead
// of 32 of (tile, 32). A forced NA (CHARSIU_GPU_QMM_NA) or PRE keeps EC = NA.
void qmm_launch_shape(const charsiu_gpu *g, uint32_t m, uint32_t tiles, uint32_t &na,
		      uint32_t &ec)
{
	na = ec = qmm_na(g, m);
	if (g->qmm_na || g->qmm_pre)
		return;
	const uint64_t sms = (uint64_t)g->sm_count;
	const uint64_t u16 = (uint64_t)tiles * ((m + 15) / 16);
	if (na == 32 && u16 > sms)
		return;
	na = 16;
	ec = 2 * u16 <= sms ? 8 : 16;
	// units of 4 activations while even they fit one round: the 2048-row
	// launches at M = 16 / 32 (32 -> 64 units) and every launch of a column
	// split's slabs (1B step at M = 16 1.266 -> 1.217 ms, M = 32 1.338 ->
	// 1.305, bit-exact; an L2 prefetch of the weight segments two stages
	// ahead measured slower on top of it)
	if (ec == 8 && 4 * u16 <= sms)
		ec = 4;
}

// The driver's tensor-map encoder, looked up once (null if the driver has none).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder()
{
	static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
		void *f = nullptr;
		cudaDriverEntryPointQueryResult res;
		if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000,
						     cudaEnableDefault, &res) != cudaSuccess ||
		    res != cudaDriverEntryPointSuccess)
			f = nullptr;
		return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
	}();
	return fn;
}

// The batched matvec's two activation boxes a stage, straight from q int8
// [m][nb*32] and d f32 [m][nb]: q viewed as (16 bytes, m rows, 2*nb chunks)
// with a box of (16, na, 32) lands as [32 chunks][na rows][16 B], the MMA's
// core matrices; d as (nb, m) with a box of (16, na) lands as [na][16]. Out
// of range reads zero, as the packing writes. false: not describable (q or d
// not 16-byte aligned, a row of d not a multiple of 16 bytes, no encoder).
bool qmm_act_maps(const int8_t *q, const float *d, uint32_t m, uint32_t nb, uint32_t na,
		  CUtensorMap *qmap, CUtensorMap *dmap)
{
	const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
	if (!enc || ((uintptr_t)q & 15) || ((uintptr_t)d & 15) || (nb * 4) % 16 || !m)
		return false;
	const cuuint32_t ones[3] = {1, 1, 1};
	const cuuint64_t qdim[3] = {16, m, (cuuint64_t)nb * 2};
	const cuuint64_t qstride[2] = {(cuuint64_t)nb * 32, 16};
	const cuuint32_t qbox[3] = {16, na, 2 * SB};
	const cuuint64_t ddim[2] = {nb, m};
	const cuuint64_t dstride[1] = {(cuuint64_t)nb * 4};
	const cuuint32_t dbox[2] = {SB, na};
	return enc(qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t *>(q), qdim, qstride,
		   qbox, ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
		   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS &&
	       enc(dmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(d), ddim, dstride,
		   dbox, ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
		   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t qmm_pack_bytes(uint32_t na, uint32_t m, uint32_t nb)
{
	return (size_t)((m + na - 1) / na) * nsegments(nb) * qmm_act_seg_bytes(na);
}

// pack_always: lay the activations out in `pack` even where the tensor copies
// could read them from q and d (the allocation-free call keeps them in its
// static array).
int launch_qmm(charsiu_gpu *g, const int *ids, unsigned n, const int8_t *q, const float *d,
	       uint32_t m, float *const *ys, uint8_t *pack, cudaStream_t st,
	       const QmmGather *gth = nullptr, bool pack_always = false)
{
	if (!n || n > (unsigned)QMM_MAX_TENSORS)
		return -1;
	uint32_t tiles = 0;
	for (unsigned i = 0; i < n; i++)
		tiles += (g->ent[ids[i]].groups + QMM_TILE_GROUPS - 1) / QMM_TILE_GROUPS;
	uint32_t na, ec;
	qmm_launch_shape(g, m, tiles, na, ec);
	const uint32_t nb = g->ent[ids[0]].nb;
	const uint32_t mt = (m + na - 1) / na, nseg = nsegments(nb);
	cudaLaunchAttribute attr[1];
	attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	attr[0].val.programmaticStreamSerializationAllowed = 1;

	QmmParams p = {};
	p.use_map = !pack_always && qmm_act_maps(q, d, m, nb, na, &p.qmap, &p.dmap) ? 1u : 0u;
	if (!p.use_map) {
		const uint64_t items = (uint64_t)mt * nseg * (SB * 2 * na + SB * na);
		cudaLaunchConfig_t pc = {};
		pc.gridDim = dim3((unsigned)((items + 255) / 256));
		pc.blockDim = dim3(256);
		pc.stream = st;
		pc.attrs = attr;
		pc.numAttrs = g->no_pdl ? 0 : 1;
		if (cudaLaunchKernelEx(&pc, qmm_pack_kernel, q, d, m, nb, na, pack) != cudaSuccess)
			return -1;
		g->launches++;
	}

	uint32_t tile_end = 0;
	for (unsigned i = 0; i < n; i++) {
		const Ent &e = g->ent[ids[i]];
		p.t[i].w = e.data;
		p.t[i].y = ys[i];
		p.t[i].rows = (uint32_t)e.rows;
		p.t[i].groups = e.groups;
		tile_end += (e.groups + QMM_TILE_GROUPS - 1) / QMM_TILE_GROUPS;
		p.t[i].tile_end = tile_end;
	}
	p.act = pack;
	p.ntensor = n;
	p.tiles = tiles;
	p.atiles = mt;
	p.nb = nb;
	p.m = m;
	p.one = 1.0f;
	p.err = g->d_err;
	if (!tiles)
		return 0;
	const bool pre = g->qmm_pre && ec == na;
	const void *fn = na == 32 ? (pre ? (const void *)qmm_tc_kernel<32, 32, true>
					 : (const void *)qmm_tc_kernel<32, 32, false>)
			 : ec == 4 ? (const void *)qmm_tc_kernel<16, 4, false>
			 : ec == 8 ? (const void *)qmm_tc_kernel<16, 8, false>
				   : (pre ? (const void *)qmm_tc_kernel<16, 16, true>
					  : (const void *)qmm_tc_kernel<16, 16, false>);
	// smem_set slots: 20..23 (NA, PRE), 19 the 8-activation slices, 18 the 4-activation
	const int slot = ec == 4 ? 18 : ec == 8 ? 19 : 20 + (na == 32 ? 2 : 0) + (pre ? 1 : 0);
	const size_t smem = qmm_smem_bytes(na, ec);
	if (!g->smem_set[slot]) {
		if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
					 (int)smem) != cudaSuccess)
			return -1;
		g->smem_set[slot] = true;
	}
	const uint32_t units = tiles * mt * (na / ec);
	cudaLaunchConfig_t cfg = {};
	cfg.gridDim = dim3(units < (uint32_t)g->sm_count ? units : (uint32_t)g->sm_count);
	cfg.blockDim = dim3(qmm_threads((int)ec));
	cfg.dynamicSmemBytes = smem;
	cfg.stream = st;
	cfg.attrs = attr;
	cfg.numAttrs = g->no_pdl ? 0 : 1;
	QmmGather garg = gth ? *gth : QmmGather{};
	void *args[2] = {&p, &garg};
	if (cudaLaunchKernelExC(&cfg, fn, args) != cudaSuccess)
		return -1;
	g->launches++;
	return 0;
}

// Activations a CUDA-core launch takes: 8, 4 or 2 while that many are left
// and their term buffers fit shared memory, else 1.
unsigned qmvm_chunk(unsigned left, uint32_t nb)
{
	for (unsigned c : {8u, 4u, 2u})
		if (left >= c && qmvm_smem_bytes((int)c, nb) <= QMV_SMEM_MAX)
			return c;
	return 1;
}

// One launch per quant type present among ids (the M = 1 kernel takes one
// type a launch; a decode's groups are always a single type).
// q6_K: q6k_kernel<W, U>, one launch a tensor: W = 4 warps at K <= 2048
// (U = 1 to K = 1024), 8 to K = 4096, 16 beyond; 8-row groups over the grid.
int launch_q6k(charsiu_gpu *g, const Ent &e, float *y, const int8_t *q, const float *d,
	       cudaStream_t st)
{
	Q6kParams p;
	p.w = e.data;
	p.y = y;
	p.rows = (uint32_t)e.rows;
	p.nsb = (uint32_t)(e.k / 256);
	p.q = q;
	p.d = d;
	if (!p.rows)
		return 0;
	static const void *const fns[4] = {
		(const void *)q6k_kernel<4, 1>, (const void *)q6k_kernel<4, 2>,
		(const void *)q6k_kernel<8, 2>, (const void *)q6k_kernel<16, 2>};
	static const int warps[4] = {4, 4, 8, 16};
	const int si = p.nsb <= 4 ? 0 : p.nsb <= 8 ? 1 : p.nsb <= 16 ? 2 : 3;
	const void *fn = fns[si];
	const int slot = 4 + si;          // 4..7
	const unsigned threads = (unsigned)warps[si] * 32;
	const size_t smem = q6k_smem_bytes(p.nsb);
	if (smem > QMV_SMEM_MAX)
		return -1;
	if (!g->smem_set[slot]) {
		if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
					 (int)QMV_SMEM_MAX) != cudaSuccess)
			return -1;
		g->smem_set[slot] = true;
	}
	const uint64_t key = (uint64_t)slot << 32 | p.nsb;
	int occ = 0;
	for (const auto &kv : g->occ)
		if (kv.first == key)
			occ = kv.second;
	if (!occ) {
		if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, (int)threads, smem) !=
			    cudaSuccess || occ < 1)
			return -1;
		g->occ.emplace_back(key, occ);
	}
	const unsigned groups = (p.rows + RG - 1) / RG;
	unsigned grid = (unsigned)occ * g->sm_count;
	if (groups < grid)
		grid = groups;
	cudaLaunchConfig_t cfg = {};
	cfg.gridDim = dim3(grid);
	cfg.blockDim = dim3(threads);
	cfg.dynamicSmemBytes = smem;
	cfg.stream = st;
	cudaLaunchAttribute attr[1];
	attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	attr[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = attr;
	cfg.numAttrs = g->no_pdl ? 0 : 1;
	void *args[1] = {&p};
	if (cudaLaunchKernelExC(&cfg, fn, args) != cudaSuccess)
		return -1;
	g->launches++;
	return 0;
}

int launch_matvec1(charsiu_gpu *g, const int *ids, unsigned n, float *const *ys, uint32_t k,
		   const int8_t *q, const float *d, cudaStream_t st)
{
	for (unsigned i = 0; i < n; i++)
		if (g->ent[ids[i]].type == TYPE_Q6_K && launch_q6k(g, g->ent[ids[i]], ys[i], q, d, st))
			return -1;
	for (uint32_t type : {TYPE_Q8_0, TYPE_Q4_0}) {    // q6_K: above
		int sub[QMV_MAX_TENSORS];
		float *sy[QMV_MAX_TENSORS];
		unsigned ns = 0;
		for (unsigned i = 0; i < n; i++)
			if (g->ent[ids[i]].type == type) {
				sub[ns] = ids[i];
				sy[ns++] = ys[i];
			}
		if (!ns)
			continue;
		QmvParams p;
		fill_params(g, p, sub, ns, sy, k, q, d);
		if (launch_qmv(g, 1, p, st))
			return -1;
	}
	return 0;
}

int check_ids(charsiu_gpu *g, const int *ids, unsigned n, unsigned k)
{
	if (!n || n > QMV_MAX_TENSORS)
		return -1;
	for (unsigned i = 0; i < n; i++) {
		if (ids[i] < 0 || (unsigned)ids[i] >= g->ent.size())
			return -1;
		if (g->ent[ids[i]].k != k) {
			whine(g, "the activation is not this tensor's K (%u vs %llu)", k,
			      (unsigned long long)g->ent[ids[i]].k);
			return -1;
		}
	}
	return 0;
}

// Queue the kernels of one host call: one launch per chunk of at most
// QMV_MAX_M activation rows (qmvm_chunk; the M = 1 path one launch per quant
// type), unless the batch goes to the tensor cores.
int queue_matvec_kernels(charsiu_gpu *g, const int *ids, unsigned n, unsigned k, unsigned m)
{
	const uint32_t nb = k / 32;
	const int8_t *dq = reinterpret_cast<const int8_t *>(g->d_act);
	const float *dd = reinterpret_cast<const float *>(g->d_act + (size_t)m * nb * 32);
	if (m >= g->qmm_min_m) {
		// q8_0 on the tensor cores; q4_0 on the CUDA cores below
		bool all_q8 = true;
		for (unsigned i = 0; i < n; i++)
			all_q8 = all_q8 && g->ent[ids[i]].type == TYPE_Q8_0;
		if (all_q8) {
			float *yd[QMV_MAX_TENSORS];
			size_t off = 0;
			for (unsigned i = 0; i < n; i++) {
				yd[i] = g->d_y + off;
				off += (size_t)m * g->ent[ids[i]].rows;
			}
			return launch_qmm(g, ids, n, dq, dd, m, yd, g->d_pack, g->stream);
		}
	}
	// the CUDA cores: each quant type its own launches (a kernel takes one);
	// q6_K one activation at a time
	size_t base[QMV_MAX_TENSORS];
	size_t off = 0;
	for (unsigned i = 0; i < n; i++) {
		base[i] = off;
		off += (size_t)m * g->ent[ids[i]].rows;
	}
	for (uint32_t type : {TYPE_Q8_0, TYPE_Q4_0, TYPE_Q6_K}) {
		int sub[QMV_MAX_TENSORS];
		size_t sbase[QMV_MAX_TENSORS];
		unsigned ns = 0;
		for (unsigned i = 0; i < n; i++)
			if (g->ent[ids[i]].type == type) {
				sub[ns] = ids[i];
				sbase[ns++] = base[i];
			}
		if (!ns)
			continue;
		for (unsigned m0 = 0, mc = 0; m0 < m; m0 += mc) {
			mc = type == TYPE_Q6_K ? 1 : qmvm_chunk(m - m0, nb);
			float *yd[QMV_MAX_TENSORS];
			for (unsigned i = 0; i < ns; i++)
				yd[i] = g->d_y + sbase[i] + (size_t)m0 * g->ent[sub[i]].rows;
			QmvParams p;
			fill_params(g, p, sub, ns, yd, k, dq + (size_t)m0 * nb * 32,
				    dd + (size_t)m0 * nb);
			const int rc = mc == 1 ? launch_matvec1(g, sub, ns, yd, k, p.q, p.d, g->stream)
					       : launch_qmv(g, (int)mc, p, g->stream);
			if (rc)
				return -1;
		}
	}
	return 0;
}

// Spin until a direct call's kernel raises the sequence flag (mapped host
// memory), under the reference's budget (src/npudev.c:560-573) as finish()
// applies it: a CUDA error, a launch that finished without signalling or one
// that never finishes retires the layer, and three slow calls in a row too.
static_assert(QMV_MAX_TENSORS <= ParCopy::MAX_SEG, "a launch group's outputs in one copy");

// The layer's large copies on its host threads: the pool the decode loop
// lent it, else one of its own made at the first copy of 64 KB or more.
void par_copy(charsiu_gpu *g, ParCopy &pc)
{
	if (pc.total >= 4 * ParCopy::CHUNK && !g->copy_pool_tried) {
		g->copy_pool_tried = true;
		const char *e = getenv("CHARSIU_GPU_THREADS");
		const long cpus = sysconf(_SC_NPROCESSORS_ONLN);
		const int threads = e ? atoi(e) : (int)(cpus > 2 ? (cpus - 1 < 8 ? cpus - 1 : 8) : 0);
		g->copy_pool = pool_new(threads);      // NULL: the caller copies alone
		g->copy_pool_owned = g->copy_pool != nullptr;
	}
	pc.run(g->copy_pool);
}

int wait_direct(charsiu_gpu *g, uint32_t seq, double t0, double mb, unsigned k)
{
	// the reference's budget (src/npudev.c:560-573), as finish() applies it
	const double budget = g->slow_us + mb * 1000.0;
	for (uint64_t spins = 1; g->h_flag[0] != seq; spins++) {
		if (spins & 1023)
			continue;
		const double el = now_us() - t0;
		if (el <= budget)
			continue;
		const cudaError_t e = cudaStreamQuery(g->stream);
		if (e != cudaSuccess && e != cudaErrorNotReady) {
			whine(g, "CUDA error %s (K=%u)", cudaGetErrorString(e), k);
			retire(g, "a CUDA error");
			return -1;
		}
		if (e == cudaSuccess && g->h_flag[0] != seq) {
			whine(g, "a call finished without signalling (K=%u)", k);
			retire(g, "a call finished without signalling");
			return -1;
		}
		if (el > budget + 10e6) {
			whine(g, "a call did not finish (K=%u)", k);
			retire(g, "it stopped answering");
			return -1;
		}
	}
	std::atomic_thread_fence(std::memory_order_acquire);
	const double t2 = now_us();
	if (*g->h_err) {
		*g->h_err = 0;
		whine(g, "a kernel wait gave up (K=%u)", k);
		retire(g, "a kernel wait gave up");
		return -1;
	}
	double took = t2 - t0;
	if (injected(g, 2))
		took = budget + 1.0;
	if (took > budget) {
		if (++g->strikes >= 3) {
			whine(g, "three slow calls in a row (K=%u)", k);
			retire(g, "it stopped answering in time");
			return -1;
		}
	} else {
		g->strikes = 0;
	}
	return 0;
}

// The direct host call, for one activation against tensors of one quant type
// (every call charsiu's decode makes): the activation travels inside the
// launch's own parameters (qmv1_inline_kernel), the matvec writes every y
// straight into mapped host memory, and its last CTA raises a sequence flag
// there, which the host spins on. One launch; no copy-engine transfer, graph
// or event sits in the call.
int run_direct(charsiu_gpu *g, const int *ids, unsigned n, const int8_t *q, const float *d,
	       unsigned k, double mb, float **ys, double t0)
{
	float *y_dev = dev_view(g->h_y);
	if (!y_dev) {
		whine(g, "a staging buffer has no device address");
		return -1;
	}
	const uint32_t nb = k / 32;
	float *yd[QMV_MAX_TENSORS];
	size_t off = 0;
	for (unsigned i = 0; i < n; i++) {
		yd[i] = y_dev + off;
		off += g->ent[ids[i]].rows;
	}
	const uint32_t seq = ++g->seq ? g->seq : ++g->seq;     // never 0, the flag's reset value
	QmvInline<QMV_INLINE_MAX_WORDS> &a = *g->inl;
	fill_params(g, a.p, ids, n, yd, k, nullptr, nullptr);
	a.p.done_count = g->d_sync;
	a.p.done_flag = g->d_flag;
	a.p.t_start = reinterpret_cast<unsigned long long *>(g->d_sync + 2);
	a.p.seq = seq;
	uint8_t *words = reinterpret_cast<uint8_t *>(a.act);
	memcpy(words, q, (size_t)nb * 32);
	memcpy(words + (size_t)nb * 32, d, (size_t)nb * sizeof(float));
	bool ok = !launch_qmv(g, 1, a.p, g->stream, &a);
	if (!ok) {
		whine(g, "the launch failed: %s", cudaGetErrorString(cudaGetLastError()));
		retire(g, "a launch failed");
		return -1;
	}
	const double t1 = now_us();
	if (wait_direct(g, seq, t0, mb, k))
		return -1;
	const double t2 = now_us();
	{
		ParCopy pc;
		off = 0;
		for (unsigned i = 0; i < n; i++) {
			const size_t cnt = g->ent[ids[i]].rows;
			pc.add(ys[i], g->h_y + off, cnt * sizeof(float));
			off += cnt;
		}
		par_copy(g, pc);
	}
	const double t3 = now_us();
	g->calls++;
	g->weight_mb += mb;
	g->h2d_us += t1 - t0;
	g->kern_ms += g->h_flag[1] * 1e-6;
	g->d2h_us += t3 - t2;
	g->busy_us += t3 - t0;
	return 0;
}

// The host-pointer matvec (charsiu_gpu_matvec / _group / _batch): the
// activation copied in as one [q | d] block, the kernels, every y copied
// back, one fence. From its second call on, a given single-activation call
// (same tensors) replays a CUDA graph of the whole sequence, so a call costs
// one graph launch and one event wait.
int run_matvec(charsiu_gpu *g, const int *ids, unsigned n, const int8_t *q, const float *d,
	       unsigned k, unsigned m, float **ys)
{
	g->call_no++;
	if (g->dead) {
		whine(g, "the GPU path is already retired");
		return -1;
	}
	if (!q || !d || !ys || !m || k % 32 || check_ids(g, ids, n, k))
		return -1;
	if (injected(g, 1)) {
		whine(g, "the launch failed (injected, K=%u)", k);
		retire(g, "a launch failed");
		return -1;
	}
	const uint32_t nb = k / 32;
	const size_t qbytes = (size_t)m * nb * 32, abytes = qbytes + (size_t)m * nb * sizeof(float);
	const size_t abytes16 = (abytes + 15) & ~(size_t)15;    // the copy-in moves 16-byte words
	size_t ytot = 0;
	double mb = 0;
	for (unsigned i = 0; i < n; i++) {
		ytot += (size_t)m * g->ent[ids[i]].rows;
		mb += g->ent[ids[i]].weight_mb;
	}
	const size_t caps[4] = {g->cap_dact, g->cap_hact, g->cap_dy, g->cap_hy};
	if (!grow_dev(g->d_act, g->cap_dact, abytes16) || !grow_host(g->h_act, g->cap_hact, abytes16) ||
	    !grow_dev(g->d_y, g->cap_dy, ytot) || !grow_host(g->h_y, g->cap_hy, ytot)) {
		whine(g, "a staging buffer would not allocate");
		return -1;
	}
	if (caps[0] != g->cap_dact || caps[1] != g->cap_hact || caps[2] != g->cap_dy ||
	    caps[3] != g->cap_hy)
		drop_graphs(g);         // they name the old staging buffers
	if (m > 1 && !grow_dev(g->d_pack, g->cap_pack, qmm_pack_bytes(qmm_na(g, m), m, nb))) {
		whine(g, "a staging buffer would not allocate");
		return -1;
	}

	const double t0 = now_us();
	if (g->direct && m == 1 && (size_t)nb * 36 <= sizeof(g->inl->act) &&
	    g->ent[ids[0]].type != TYPE_Q6_K) {
		bool one_type = true;
		for (unsigned i = 1; i < n; i++)
			one_type = one_type && g->ent[ids[i]].type == g->ent[ids[0]].type;
		if (one_type)
			return run_direct(g, ids, n, q, d, k, mb, ys, t0);
	}
	memcpy(g->h_act, q, qbytes);
	memcpy(g->h_act + qbytes, d, (size_t)m * nb * sizeof(float));

	CallGraph *cg = nullptr;
	if (m == 1) {
		for (CallGraph &c : g->graphs)
			if (c.n == n && c.k == k && !memcmp(c.ids, ids, n * sizeof(int)))
				cg = &c;
	}
	bool ok = true;
	if (cg && cg->exec) {
		ok = cudaGraphLaunch(cg->exec, g->stream) == cudaSuccess;
	} else {
		// the first call of a set runs eagerly (warming every launch cache)
		// and records the set; the second captures it
		cudaGraph_t graph = nullptr;
		const bool capture = cg != nullptr;
		if (capture)
			ok = cudaStreamBeginCapture(g->stream, cudaStreamCaptureModeThreadLocal) ==
			     cudaSuccess;
		ok = ok && cudaMemcpyAsync(g->d_act, g->h_act, abytes, cudaMemcpyHostToDevice,
					   g->stream) == cudaSuccess;
		// while capturing, external records, so the graph holds real event
		// nodes (a plain record there is only a dependency edge)
		const unsigned rf = capture ? cudaEventRecordExternal : cudaEventRecordDefault;
		ok = ok && cudaEventRecordWithFlags(g->ev_k0, g->stream, rf) == cudaSuccess;
		ok = ok && !queue_matvec_kernels(g, ids, n, k, m);
		ok = ok && cudaEventRecordWithFlags(g->ev_k1, g->stream, rf) == cudaSuccess;
		ok = ok && cudaMemcpyAsync(g->h_y, g->d_y, ytot * sizeof(float),
					   cudaMemcpyDeviceToHost, g->stream) == cudaSuccess;
		if (capture) {
			ok = cudaStreamEndCapture(g->stream, &graph) == cudaSuccess && ok;
			ok = ok && cudaGraphInstantiate(&cg->exec, graph, 0) == cudaSuccess;
			if (graph)
				cudaGraphDestroy(graph);
			ok = ok && cudaGraphLaunch(cg->exec, g->stream) == cudaSuccess;
		} else if (m == 1 && n <= QMV_MAX_TENSORS && g->graphs.size() < 4 * g->max_tensors) {
			CallGraph c = {};
			c.n = n;
			c.k = k;
			memcpy(c.ids, ids, n * sizeof(int));
			g->graphs.push_back(c);
		}
	}
	if (!ok) {
		whine(g, "the launch failed: %s", cudaGetErrorString(cudaGetLastError()));
		retire(g, "a launch failed");
		return -1;
	}
	cudaEventRecord(g->ev_done, g->stream);
	const double t1 = now_us();
	if (finish(g, t0, mb, k, (unsigned)g->ent[ids[0]].n))
		return -1;
	const double t2 = now_us();
	size_t off = 0;
	for (unsigned i = 0; i < n; i++) {
		const size_t cnt = (size_t)m * g->ent[ids[i]].rows;
		memcpy(ys[i], g->h_y + off, cnt * sizeof(float));
		off += cnt;
	}
	float kms = 0;
	if (cudaEventElapsedTime(&kms, g->ev_k0, g->ev_k1) != cudaSuccess) {
		kms = 0;
		cudaGetLastError();      // timing is best effort; clear it
	}
	const double t3 = now_us();
	g->calls++;
	g->weight_mb += mb;
	g->h2d_us += t1 - t0;
	g->kern_ms += kms;
	g->d2h_us += t3 - t2;
	g->busy_us += t3 - t0;
	return 0;
}

} // namespace

// ---- what the decode step (decoder.cu) asks of the layer ------------------------

namespace cgpu {

int layer_device(const charsiu_gpu *g)
{
	return g->device;
}

bool layer_no_pdl(const charsiu_gpu *g)
{
	return g->no_pdl != 0;
}

bool layer_whole(const charsiu_gpu *g)
{
	return g->world == 1;
}

// K, rows and quant type of tensor id; false for an unknown id
bool layer_tensor(const charsiu_gpu *g, int id, uint64_t *k, uint64_t *rows, uint32_t *type)
{
	if (id < 0 || (size_t)id >= g->ent.size())
		return false;
	*k = g->ent[id].k;
	*rows = g->ent[id].rows;
	*type = g->ent[id].type;
	return true;
}

void layer_whine(charsiu_gpu *g, const char *why)
{
	whine(g, "%s", why);
}

} // namespace cgpu

// ---- scratch for charsiu_gpu_matvec_batch_noalloc -----------------------------
//
// For callers that cannot allocate device memory while they run, the batched
// tensor-core matvec can keep its packed activation tiles here instead of in
// the layer's staging buffer (which is grown with cudaMalloc on first use).
// A fixed 1 MiB: every GPU that loads this library holds it until exit.
static constexpr size_t NOALLOC_SCRATCH_BYTES = (size_t)1 << 20;
static __device__ __align__(256) uint8_t noalloc_scratch[NOALLOC_SCRATCH_BYTES];

// In host code `noalloc_scratch` is only a stand-in for the device array, so
// its device address is looked up (with the layer's device current) by each
// layer's first allocation-free call and kept in that layer: a layer opened
// after a device reset looks it up afresh, and no table is shared between
// threads.
static uint8_t *noalloc_scratch_of(charsiu_gpu *g)
{
	if (!g->noalloc_scratch) {
		void *ptr = nullptr;
		if (cudaGetSymbolAddress(&ptr, noalloc_scratch) != cudaSuccess) {
			cudaGetLastError();
			return nullptr;
		}
		g->noalloc_scratch = static_cast<uint8_t *>(ptr);
	}
	return g->noalloc_scratch;
}

extern "C" {

struct charsiu_gpu *charsiu_gpu_open_ex(unsigned max_k, unsigned max_n, unsigned max_tensors,
					int device, unsigned rank, unsigned world)
{
	int ndev = 0;
	if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
		fprintf(stderr, "charsiu: no CUDA device %d\n", device);
		return nullptr;
	}
	// the widest activation every kernel's shared-memory plan holds
	if (!world || rank >= world || !max_k || max_k % 32 || max_k > MAX_K || !max_tensors)
		return nullptr;
	cudaDeviceProp prop;
	if (cudaSetDevice(device) != cudaSuccess ||
	    cudaGetDeviceProperties(&prop, device) != cudaSuccess)
		return nullptr;
	if (prop.major != 10 || prop.minor != 0) {
		fprintf(stderr, "charsiu: device %d is sm_%d%d; this build is sm_100a only\n",
			device, prop.major, prop.minor);
		return nullptr;
	}
	charsiu_gpu *g = new charsiu_gpu;
	g->device = device;
	g->rank = rank;
	g->world = world;
	g->max_k = max_k;
	g->max_n = max_n;
	g->max_tensors = max_tensors;
	g->sm_count = prop.multiProcessorCount;
	g->slow_us = (double)env_u("CHARSIU_GPU_SLOW_US", 100000);
	g->no_pdl = getenv("CHARSIU_GPU_NO_PDL") != nullptr;
	if (const char *e = getenv("CHARSIU_GPU_PDL_EARLY"))
		g->pdl_early = atoi(e) != 0;
	if (const char *e = getenv("CHARSIU_GPU_GATHER_PDL"))
		g->gather_pdl = atoi(e) != 0;
	if (const char *dir = getenv("CHARSIU_GPU_DIRECT"))
		g->direct = strcmp(dir, "0") != 0;
	if (const char *na = getenv("CHARSIU_GPU_QMM_NA"))
		g->qmm_na = !strcmp(na, "16") ? 16 : !strcmp(na, "32") ? 32 : 0;
	if (const char *mm = getenv("CHARSIU_GPU_QMM_MIN_M"))
		g->qmm_min_m = atoi(mm) > 2 ? (uint32_t)atoi(mm) : 2;
	if (const char *pre = getenv("CHARSIU_GPU_QMM_PRE"))
		g->qmm_pre = !strcmp(pre, "1");
	g->ent.reserve(max_tensors);
	if (cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking) != cudaSuccess ||
	    cudaEventCreate(&g->ev_k0) != cudaSuccess || cudaEventCreate(&g->ev_k1) != cudaSuccess ||
	    cudaEventCreateWithFlags(&g->ev_done, cudaEventDisableTiming) != cudaSuccess ||
	    cudaHostAlloc((void **)&g->h_err, sizeof(int), cudaHostAllocMapped) != cudaSuccess ||
	    cudaHostGetDevicePointer((void **)&g->d_err, (void *)g->h_err, 0) != cudaSuccess ||
	    cudaHostAlloc((void **)&g->h_flag, 4 * sizeof(uint32_t), cudaHostAllocMapped) !=
		    cudaSuccess ||
	    cudaHostGetDevicePointer((void **)&g->d_flag, (void *)g->h_flag, 0) != cudaSuccess ||
	    cudaMalloc((void **)&g->d_sync, 4 * sizeof(uint32_t)) != cudaSuccess ||
	    cudaMemset(g->d_sync, 0, 4 * sizeof(uint32_t)) != cudaSuccess) {
		charsiu_gpu_close(g);
		return nullptr;
	}
	const size_t nb = max_k / 32;
	*g->h_err = 0;
	for (int i = 0; i < 4; i++)
		g->h_flag[i] = 0;
	g->inl = new (std::nothrow) QmvInline<QMV_INLINE_MAX_WORDS>();
	if (!g->inl) {
		charsiu_gpu_close(g);
		return nullptr;
	}
	if (!grow_dev(g->d_act, g->cap_dact, nb * 36 + 16) ||
	    !grow_host(g->h_act, g->cap_hact, nb * 36 + 16) ||
	    !grow_dev(g->d_y, g->cap_dy, (size_t)max_n + 64) ||
	    !grow_host(g->h_y, g->cap_hy, (size_t)max_n + 64)) {
		charsiu_gpu_close(g);
		return nullptr;
	}
	return g;
}

struct charsiu_gpu *charsiu_gpu_open(unsigned max_k, unsigned max_n, unsigned max_tensors)
{
	return charsiu_gpu_open_ex(max_k, max_n, max_tensors, 0, 0, 1);
}

void charsiu_gpu_close(struct charsiu_gpu *g)
{
	if (!g)
		return;
	cudaSetDevice(g->device);
	if (!g->dead && g->stream)
		cudaStreamSynchronize(g->stream);
	for (Ent &e : g->ent)
		if (e.data)
			cudaFree(e.data);
	drop_graphs(g);
	cudaFree(g->d_act);
	cudaFree(g->d_q);
	cudaFree(g->d_pack);
	cudaFree(g->d_y);
	cudaFree(g->d_i8);
	cudaFree(g->d_dots);
	if (g->h_err)
		cudaFreeHost((void *)g->h_err);
	if (g->h_flag)
		cudaFreeHost((void *)g->h_flag);
	delete g->inl;
	delete g->i8inl;
	if (g->copy_pool_owned)
		pool_free(g->copy_pool);
	cudaFree(g->d_sync);
	cudaFree(g->d_gather_count);
	cudaFreeHost(g->h_act);
	cudaFreeHost(g->h_y);
	cudaFreeHost(g->h_i8);
	if (g->ev_k0)
		cudaEventDestroy(g->ev_k0);
	if (g->ev_k1)
		cudaEventDestroy(g->ev_k1);
	if (g->ev_done)
		cudaEventDestroy(g->ev_done);
	if (g->stream)
		cudaStreamDestroy(g->stream);
	delete g;
}

int charsiu_gpu_add_blocks(struct charsiu_gpu *g, uint32_t type, uint64_t k, uint64_t n,
			   const void *blocks, const char *name)
{
	if (!g)
		return -1;
	g->call_no++;
	if (g->dead) {
		whine(g, "the GPU path is already retired");
		return -1;
	}
	if (type != TYPE_Q8_0 && type != TYPE_Q4_0 && type != TYPE_Q6_K) {
		whine(g, "type %u is not q8_0, q4_0 or q6_K (%s)", type, name ? name : "?");
		return -1;
	}
	const uint32_t kunit = type == TYPE_Q6_K ? 256 : 32;
	if (!blocks || !k || k % kunit || !n || k > g->max_k) {
		whine(g, "K=%llu is not a multiple of %u within the opened maximum (%s)",
		      (unsigned long long)k, kunit, name ? name : "?");
		return -1;
	}
	if (n > g->max_n) {
		whine(g, "wider than the device was opened for (N=%llu, %s)",
		      (unsigned long long)n, name ? name : "?");
		return -1;
	}
	if (g->ent.size() >= g->max_tensors) {
		whine(g, "no tensor slots left");
		return -1;
	}
	cudaSetDevice(g->device);
	cudaGetLastError();              // a stale error must not be read as this upload's

	Ent e;
	memset(&e, 0, sizeof(e));
	snprintf(e.name, sizeof(e.name), "%s", name ? name : "");
	e.type = type;
	e.k = k;
	e.n = n;
	e.nb = (uint32_t)(k / 32);
	const uint64_t gtot = (n + RG - 1) / RG;
	const uint64_t per = (gtot + g->world - 1) / g->world;
	const uint64_t g0 = per * g->rank, g1 = g0 + per < gtot ? g0 + per : gtot;
	e.row0 = g0 * RG < n ? g0 * RG : n;
	const uint64_t rend = g1 * RG < n ? g1 * RG : n;
	e.rows = rend > e.row0 ? rend - e.row0 : 0;
	e.groups = (uint32_t)((e.rows + RG - 1) / RG);
	const bool q6 = type == TYPE_Q6_K;
	const uint32_t nsb = (uint32_t)(k / 256);
	e.bytes = q6 ? (size_t)e.rows * q6k_row_bytes(nsb) : (size_t)e.groups * group_bytes(type, e.nb);
	const uint64_t rb = q6 ? (uint64_t)nsb * 210 : (uint64_t)e.nb * (quant_bytes(type) + 2);
	e.weight_mb = (double)e.rows * rb / 1e6;

	if (injected(g, 3) || (e.bytes && cudaMalloc(&e.data, e.bytes) != cudaSuccess)) {
		e.data = nullptr;
		whine(g, "a weight buffer would not allocate (%s, %.1f MB)", e.name, e.bytes / 1e6);
		return -1;
	}
	if (e.bytes) {
		uint8_t *stage = nullptr;
		const uint64_t chunk_rows = ((64ull << 20) / rb) & ~(uint64_t)(RG - 1);
		const uint64_t cr = chunk_rows ? chunk_rows : RG;
		const size_t sbytes = (size_t)(cr < e.rows ? cr : e.rows) * rb;
		bool ok = cudaMemsetAsync(e.data, 0, e.bytes, g->stream) == cudaSuccess &&
			  cudaMalloc(&stage, sbytes) == cudaSuccess;
		const uint8_t *src = static_cast<const uint8_t *>(blocks) + e.row0 * rb;
		for (uint64_t r0 = 0; ok && r0 < e.rows; r0 += cr) {
			const uint64_t nr = e.rows - r0 < cr ? e.rows - r0 : cr;
			ok = cudaMemcpyAsync(stage, src + r0 * rb, nr * rb, cudaMemcpyHostToDevice,
					     g->stream) == cudaSuccess;
			if (q6) {
				const uint64_t thr = nr * nsb;
				q6k_repack_kernel<<<(unsigned)((thr + 255) / 256), 256, 0, g->stream>>>(
					stage, nsb, (uint32_t)nr, e.data + r0 * q6k_row_bytes(nsb));
			} else {
				const uint64_t thr = nr * e.nb;
				repack_kernel<<<(unsigned)((thr + 255) / 256), 256, 0, g->stream>>>(
					stage, type, e.nb, (uint32_t)r0, (uint32_t)nr, e.data);
			}
			ok = ok && cudaGetLastError() == cudaSuccess &&
			     cudaStreamSynchronize(g->stream) == cudaSuccess;
		}
		if (stage)
			cudaFree(stage);
		if (!ok) {
			cudaFree(e.data);
			whine(g, "the weight upload failed (%s)", e.name);
			return -1;
		}
	}
	g->ent.push_back(e);
	return (int)g->ent.size() - 1;
}

int charsiu_gpu_add(struct charsiu_gpu *g, const struct gguf_tensor *w)
{
	if (!g || !w)
		return -1;
	for (size_t i = 0; i < g->ent.size(); i++)
		if (g->ent[i].key == (const void *)w)
			return (int)i;
	const RefGgufTensor *t = reinterpret_cast<const RefGgufTensor *>(w);
	uint64_t rows = 1;
	for (unsigned d = 1; d < t->n_dims && d < 4; d++)
		rows *= t->ne[d];
	const int id = charsiu_gpu_add_blocks(g, t->type, t->ne[0], rows, t->data, t->name);
	if (id >= 0)
		g->ent[id].key = w;
	return id;
}

int charsiu_gpu_rows(const struct charsiu_gpu *g, int id, uint64_t *row0, uint64_t *nrows)
{
	if (!g || id < 0 || (size_t)id >= g->ent.size())
		return -1;
	if (row0)
		*row0 = g->ent[id].row0;
	if (nrows)
		*nrows = g->ent[id].rows;
	return 0;
}

int charsiu_gpu_matvec_q(struct charsiu_gpu *g, const int *ids, unsigned n, const int8_t *q,
			 const float *d, unsigned k, float **ys)
{
	if (!g)
		return -1;
	cudaSetDevice(g->device);
	return run_matvec(g, ids, n, q, d, k, 1, ys);
}

int charsiu_gpu_matvec(struct charsiu_gpu *g, int id, const struct charsiu_act *a, float *y)
{
	if (!g || !a)
		return -1;
	const RefAct *act = reinterpret_cast<const RefAct *>(a);
	if (!act->quantised) {
		whine(g, "the activation is not quantised (CHARSIU_NO_QACT?)");
		return -1;
	}
	float *ys[1] = {y};
	return charsiu_gpu_matvec_q(g, &id, 1, act->q, act->d, (unsigned)act->n, ys);
}

int charsiu_gpu_matvec_group(struct charsiu_gpu *g, const int *ids, unsigned n,
			     const struct charsiu_act *a, float **ys)
{
	if (!g || !a)
		return -1;
	const RefAct *act = reinterpret_cast<const RefAct *>(a);
	if (!act->quantised)
		return -1;
	return charsiu_gpu_matvec_q(g, ids, n, act->q, act->d, (unsigned)act->n, ys);
}

int charsiu_gpu_matvec_batch(struct charsiu_gpu *g, int id, unsigned m, const int8_t *q,
			     const float *d, unsigned k, float *y)
{
	if (!g)
		return -1;
	cudaSetDevice(g->device);
	float *ys[1] = {y};
	return run_matvec(g, &id, 1, q, d, k, m, ys);
}

int charsiu_gpu_matvec_dev(struct charsiu_gpu *g, const int *ids, unsigned n, const int8_t *q,
			   const float *d, float *const *ys, void *stream)
{
	if (!g || g->dead || !q || !d || !ys || ((uintptr_t)q & 15) || ((uintptr_t)d & 3))
		return -1;
	if (!n || n > QMV_MAX_TENSORS || ids[0] < 0 || (size_t)ids[0] >= g->ent.size())
		return -1;
	const unsigned k = (unsigned)g->ent[ids[0]].k;
	if (check_ids(g, ids, n, k))
		return -1;
	cudaSetDevice(g->device);
	return launch_matvec1(g, ids, n, ys, k, q, d, stream ? (cudaStream_t)stream : g->stream);
}

int charsiu_gpu_matvec_batch_dev(struct charsiu_gpu *g, int id, unsigned m, const int8_t *q,
				 const float *d, float *y, void *stream)
{
	if (!g || g->dead || !q || !d || !y || !m || ((uintptr_t)q & 15))
		return -1;
	if (id < 0 || (size_t)id >= g->ent.size())
		return -1;
	cudaSetDevice(g->device);
	const Ent &e = g->ent[id];
	const uint32_t nb = e.nb;
	cudaStream_t st = stream ? (cudaStream_t)stream : g->stream;
	if (m >= g->qmm_min_m && e.type == TYPE_Q8_0) {
		if (!grow_dev(g->d_pack, g->cap_pack, qmm_pack_bytes(qmm_na(g, m), m, nb)))
			return -1;
		return launch_qmm(g, &id, 1, q, d, m, &y, g->d_pack, st);
	}
	for (unsigned m0 = 0; m0 < m;) {
		const unsigned mc = e.type == TYPE_Q6_K ? 1 : qmvm_chunk(m - m0, nb);
		float *yd[1] = {y + (size_t)m0 * e.rows};
		QmvParams p;
		fill_params(g, p, &id, 1, yd, (uint32_t)e.k, q + (size_t)m0 * nb * 32,
			    d + (size_t)m0 * nb);
		if (mc == 1 ? launch_matvec1(g, &id, 1, yd, (uint32_t)e.k, p.q, p.d, st)
			    : launch_qmv(g, (int)mc, p, st))
			return -1;
		m0 += mc;
	}
	return 0;
}

int charsiu_gpu_matvec_batch_group_dev(struct charsiu_gpu *g, const int *ids, unsigned n,
				       unsigned m, const int8_t *q, const float *d, float *const *ys,
				       void *stream)
{
	if (!g || g->dead || !ids || !q || !d || !ys || !m || ((uintptr_t)q & 15) ||
	    !n || n > (unsigned)QMM_MAX_TENSORS)
		return -1;
	for (unsigned i = 0; i < n; i++)
		if (ids[i] < 0 || (size_t)ids[i] >= g->ent.size() || !ys[i] ||
		    g->ent[ids[i]].k != g->ent[ids[0]].k)
			return -1;
	cudaSetDevice(g->device);
	bool all_q8 = m >= g->qmm_min_m;
	for (unsigned i = 0; i < n; i++)
		all_q8 = all_q8 && g->ent[ids[i]].type == TYPE_Q8_0;
	if (all_q8) {
		const uint32_t nb = g->ent[ids[0]].nb;
		if (!grow_dev(g->d_pack, g->cap_pack, qmm_pack_bytes(qmm_na(g, m), m, nb)))
			return -1;
		return launch_qmm(g, ids, n, q, d, m, ys, g->d_pack,
				  stream ? (cudaStream_t)stream : g->stream);
	}
	// the CUDA cores: the tensors of each quant type in one launch a chunk of
	// activations (as queue_matvec_kernels does for host calls), each tensor's
	// y[a][rows] at its own stride; q6_K one activation at a time
	cudaStream_t st = stream ? (cudaStream_t)stream : g->stream;
	const uint32_t nb = g->ent[ids[0]].nb, k = (uint32_t)g->ent[ids[0]].k;
	for (uint32_t type : {TYPE_Q8_0, TYPE_Q4_0, TYPE_Q6_K}) {
		int sub[QMV_MAX_TENSORS];
		float *sy[QMV_MAX_TENSORS];
		unsigned ns = 0;
		for (unsigned i = 0; i < n; i++)
			if (g->ent[ids[i]].type == type) {
				sub[ns] = ids[i];
				sy[ns++] = ys[i];
			}
		if (!ns)
			continue;
		for (unsigned m0 = 0, mc = 0; m0 < m; m0 += mc) {
			mc = type == TYPE_Q6_K ? 1 : qmvm_chunk(m - m0, nb);
			float *yd[QMV_MAX_TENSORS];
			for (unsigned i = 0; i < ns; i++)
				yd[i] = sy[i] + (size_t)m0 * g->ent[sub[i]].rows;
			QmvParams p;
			fill_params(g, p, sub, ns, yd, k, q + (size_t)m0 * nb * 32, d + (size_t)m0 * nb);
			const int rc = mc == 1 ? launch_matvec1(g, sub, ns, yd, k, p.q, p.d, st)
					       : launch_qmv(g, (int)mc, p, st);
			if (rc)
				return -1;
		}
	}
	return 0;
}

// ---- the matvec fused with its all-gather (column split over GPUs) ------------

void *charsiu_gpu_ipc_alloc(struct charsiu_gpu *g, size_t bytes)
{
	if (!g || !bytes)
		return nullptr;
	cudaSetDevice(g->device);
	void *p = nullptr;
	if (cudaMalloc(&p, bytes) != cudaSuccess)
		return nullptr;
	if (cudaMemset(p, 0, bytes) != cudaSuccess) {
		cudaFree(p);
		return nullptr;
	}
	return p;
}

int charsiu_gpu_ipc_handle(struct charsiu_gpu *g, void *ptr, unsigned char *handle)
{
	if (!g || !ptr || !handle)
		return -1;
	cudaSetDevice(g->device);
	cudaIpcMemHandle_t h;
	static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
	if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess)
		return -1;
	memcpy(handle, &h, sizeof(h));
	return 0;
}

void *charsiu_gpu_ipc_open(struct charsiu_gpu *g, const unsigned char *handle)
{
	if (!g || !handle)
		return nullptr;
	cudaSetDevice(g->device);
	cudaIpcMemHandle_t h;
	memcpy(&h, handle, sizeof(h));
	void *p = nullptr;
	if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
		return nullptr;
	return p;
}

void charsiu_gpu_ipc_free(struct charsiu_gpu *g, void *ptr, int opened)
{
	if (!g || !ptr)
		return;
	cudaSetDevice(g->device);
	if (opened)
		cudaIpcCloseMemHandle(ptr);
	else
		cudaFree(ptr);
}

int charsiu_gpu_read_device(struct charsiu_gpu *g, const void *dev_ptr, void *host, size_t bytes)
{
	if (!g || !dev_ptr || !host)
		return -1;
	cudaSetDevice(g->device);
	return cudaMemcpy(host, dev_ptr, bytes, cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -1;
}

int charsiu_gpu_kernel_error(struct charsiu_gpu *g)
{
	if (!g || !g->h_err)
		return -1;
	const int e = *g->h_err;
	if (e) {
		*g->h_err = 0;
		whine(g, "a kernel wait gave up (code %d)", e);
		retire(g, "a kernel wait gave up");
	}
	return e;
}

int charsiu_gpu_matvec_batch_gather_dev(struct charsiu_gpu *g, const int *ids, unsigned n,
					unsigned m, const int8_t *q, const float *d,
					float *const *full_ys, uint32_t *const *syncs,
					unsigned signal_idx, unsigned wait_idx, unsigned wait_mult,
					int wait_adj, void *stream)
{
	if (!g || g->dead || !ids || !q || !d || !full_ys || !syncs || ((uintptr_t)q & 15) ||
	    g->world > (unsigned)QMM_MAX_RANKS || !n || n > (unsigned)QMM_MAX_TENSORS ||
	    m < g->qmm_min_m)
		return -1;
	for (unsigned i = 0; i < n; i++)
		if (ids[i] < 0 || (size_t)ids[i] >= g->ent.size() ||
		    g->ent[ids[i]].type != TYPE_Q8_0 || g->ent[ids[i]].k != g->ent[ids[0]].k)
			return -1;
	cudaSetDevice(g->device);
	QmmGather gth = {};
	for (unsigned r = 0; r < g->world; r++) {
		if (!syncs[r])
			return -1;
		gth.sync[r] = syncs[r];
		for (unsigned i = 0; i < n; i++) {
			if (!full_ys[r * n + i])
				return -1;
			gth.y[r][i] = full_ys[r * n + i];
		}
	}
	for (unsigned i = 0; i < n; i++) {
		gth.row0[i] = (uint32_t)g->ent[ids[i]].row0;
		gth.ncols[i] = (uint32_t)g->ent[ids[i]].n;
	}
	if (!g->d_gather_count) {
		if (cudaMalloc((void **)&g->d_gather_count, sizeof(uint32_t)) != cudaSuccess ||
		    cudaMemset(g->d_gather_count, 0, sizeof(uint32_t)) != cudaSuccess)
			return -1;
	}
	gth.cta_count = g->d_gather_count;
	gth.world = g->world;
	gth.rank = g->rank;
	gth.signal_idx = signal_idx;
	gth.wait_idx = wait_idx;
	gth.wait_mult = wait_mult;
	gth.wait_adj = wait_adj;
	const uint32_t nb = g->ent[ids[0]].nb;
	if (!grow_dev(g->d_pack, g->cap_pack, qmm_pack_bytes(qmm_na(g, m), m, nb)))
		return -1;
	float *unused[QMM_MAX_TENSORS] = {};
	return launch_qmm(g, ids, n, q, d, m, unused, g->d_pack,
			  stream ? (cudaStream_t)stream : g->stream, &gth);
}

int charsiu_gpu_gather_epoch_dev(struct charsiu_gpu *g, uint32_t *sync_local, void *stream)
{
	if (!g || g->dead || !sync_local)
		return -1;
	cudaSetDevice(g->device);
	cudaLaunchConfig_t cfg = {};
	cfg.gridDim = dim3(1);
	cfg.blockDim = dim3(32);
	cfg.stream = stream ? (cudaStream_t)stream : g->stream;
	cudaLaunchAttribute attr[1];
	attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	attr[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = attr;
	cfg.numAttrs = g->no_pdl || !g->gather_pdl ? 0 : 1;
	if (cudaLaunchKernelEx(&cfg, gather_epoch_kernel, sync_local) != cudaSuccess)
		return -1;
	g->launches++;
	return 0;
}

int charsiu_gpu_matvec_gather_dev(struct charsiu_gpu *g, const int *ids, unsigned n,
				  const int8_t *q, const float *d, float *const *full_ys,
				  uint32_t *const *syncs, unsigned signal_idx, unsigned wait_idx,
				  unsigned wait_mult, int wait_adj, void *stream)
{
	if (!g || g->dead || !ids || !q || !d || !full_ys || !syncs || ((uintptr_t)q & 15) ||
	    g->world > (unsigned)QMV_MAX_RANKS || !n || n > (unsigned)QMV_MAX_TENSORS)
		return -1;
	uint32_t k = 0;
	for (unsigned i = 0; i < n; i++) {
		if (ids[i] < 0 || (size_t)ids[i] >= g->ent.size())
			return -1;
		const Ent &e = g->ent[ids[i]];
		if ((i && (e.k != k || e.type != g->ent[ids[0]].type)) || e.type == TYPE_Q6_K)
			return -1;
		k = (uint32_t)e.k;
	}
	cudaSetDevice(g->device);
	QmvGather gth = {};
	for (unsigned r = 0; r < g->world; r++) {
		if (!syncs[r])
			return -1;
		gth.sync[r] = syncs[r];
		for (unsigned i = 0; i < n; i++) {
			if (!full_ys[r * n + i])
				return -1;
			gth.y[r][i] = full_ys[r * n + i];
		}
	}
	for (unsigned i = 0; i < n; i++)
		gth.row0[i] = (uint32_t)g->ent[ids[i]].row0;
	if (!g->d_gather_count) {
		if (cudaMalloc((void **)&g->d_gather_count, sizeof(uint32_t)) != cudaSuccess ||
		    cudaMemset(g->d_gather_count, 0, sizeof(uint32_t)) != cudaSuccess)
			return -1;
	}
	gth.cta_count = g->d_gather_count;
	gth.world = g->world;
	gth.rank = g->rank;
	gth.signal_idx = signal_idx;
	gth.wait_idx = wait_idx;
	gth.wait_mult = wait_mult;
	gth.wait_adj = wait_adj;
	float *unused[QMV_MAX_TENSORS] = {};
	QmvParams p;
	fill_params(g, p, ids, n, unused, k, q, d);
	return launch_qmv(g, 1, p, stream ? (cudaStream_t)stream : g->stream, nullptr, &gth);
}

// The batched q8_0 matvec with nothing allocated: the same pack and
// tensor-core kernels as charsiu_gpu_matvec_batch_dev, with the packed
// activations always laid out in noalloc_scratch (not read from q and d by
// tensor copies, as the _dev form does where it can). The pack step writes
// every byte the matmul then reads (padding zeroed), so no clearing is needed
// between calls; calls that overlap on one GPU share the array and race.
int charsiu_gpu_matvec_batch_noalloc(struct charsiu_gpu *g, int id, unsigned m, const int8_t *q,
				     const float *d, float *y, void *stream)
{
	if (!g || g->dead || !q || !d || !y || !m || ((uintptr_t)q & 15) || ((uintptr_t)d & 3))
		return -1;
	if (id < 0 || (size_t)id >= g->ent.size())
		return -1;
	const Ent &e = g->ent[id];
	if (e.type != TYPE_Q8_0) {
		whine(g, "the allocation-free batched matvec takes q8_0 tensors only (%s)", e.name);
		return -1;
	}
	const size_t need = qmm_pack_bytes(qmm_na(g, m), m, e.nb);
	if (need > NOALLOC_SCRATCH_BYTES) {
		whine(g, "the allocation-free batched matvec holds %zu bytes of packed activations; "
			 "m=%u at K=%llu needs %zu", NOALLOC_SCRATCH_BYTES, m,
		      (unsigned long long)e.k, need);
		return -1;
	}
	cudaSetDevice(g->device);
	uint8_t *scratch = noalloc_scratch_of(g);
	if (!scratch) {
		whine(g, "the allocation-free scratch has no device address on device %d", g->device);
		return -1;
	}
	return launch_qmm(g, &id, 1, q, d, m, &y, scratch,
			  stream ? (cudaStream_t)stream : g->stream, nullptr, true);
}

int charsiu_gpu_act_quantise_dev(struct charsiu_gpu *g, const float *x, unsigned m, unsigned k,
				 int8_t *q, float *d, void *stream)
{
	if (!g || g->dead || !x || !q || !d || !m || !k)
		return -1;
	cudaSetDevice(g->device);
	const uint32_t nb = (k + 31) / 32;
	const uint64_t threads = (uint64_t)m * nb * 32;
	act_quantise_kernel<<<(unsigned)((threads + 255) / 256), 256, 0,
			      stream ? (cudaStream_t)stream : g->stream>>>(x, m, k, nb, q, d);
	if (cudaGetLastError() != cudaSuccess)
		return -1;
	g->launches++;
	return 0;
}

int charsiu_gpu_row_dev(struct charsiu_gpu *g, int id, const int32_t *row, float *out,
			void *stream)
{
	if (!g || g->dead || !row || !out || id < 0 || (size_t)id >= g->ent.size())
		return -1;
	const Ent &e = g->ent[id];
	if (e.row0 != 0 || e.rows != e.n) {
		whine(g, "%s is split over GPUs; a row lookup needs all of it", e.name);
		return -1;
	}
	cudaSetDevice(g->device);
	cudaLaunchConfig_t cfg = {};
	cfg.gridDim = dim3((unsigned)((e.k + 255) / 256));
	cfg.blockDim = dim3(256);
	cfg.stream = stream ? (cudaStream_t)stream : g->stream;
	cudaLaunchAttribute attr[1];
	attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	attr[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = attr;
	cfg.numAttrs = g->no_pdl ? 0 : 1;
	if (cudaLaunchKernelEx(&cfg, row_f32_kernel, (const uint8_t *)e.data, e.type, (uint64_t)e.k,
			       (uint32_t)e.rows, row, out, g->d_err) != cudaSuccess)
		return -1;
	g->launches++;
	return 0;
}

} // extern "C"

// A small int8 job as one direct call (i8mm_simt_inline_kernel): the operands
// in the launch's own parameters, the bytes written into mapped host memory,
// the last CTA raising the sequence flag the host spins on. One launch; no
// copy-engine transfer or event sits in the call.
static int matmul_i8_direct(charsiu_gpu *g, unsigned m, unsigned k, unsigned n,
			    const uint8_t *a, const uint8_t *w, const int32_t *bias, float in_scale,
			    float wt_scale, float out_scale, int in_zp, int wt_zp, int out_zp,
			    int8_t *out)
{
	const size_t sa = (size_t)m * k, sw = (size_t)n * k, sb = (size_t)n * 4;
	const size_t ow = (sa + 15) & ~(size_t)15, ob = (ow + sw + 15) & ~(size_t)15;
	if (!g->i8inl)
		g->i8inl = new (std::nothrow) I8Inline<I8_INLINE_W2>;
	if (!g->i8inl || !grow_host(g->h_i8, g->cap_hi8, (size_t)m * n)) {
		whine(g, "a staging buffer would not allocate");
		return -1;
	}
	int8_t *out_dev = reinterpret_cast<int8_t *>(dev_view(g->h_i8));
	if (!out_dev) {
		whine(g, "a staging buffer has no device address");
		return -1;
	}
	const double t0 = now_us();
	I8Inline<I8_INLINE_W2> &x = *g->i8inl;
	uint8_t *data = reinterpret_cast<uint8_t *>(x.data);
	memcpy(data, a, sa);
	memcpy(data + ow, w, sw);
	memcpy(data + ob, bias, sb);
	const uint32_t seq = ++g->seq ? g->seq : ++g->seq;     // never 0, the flag's reset value
	x.p = I8Params{};
	x.p.a = nullptr;
	x.p.w = nullptr;
	x.p.bias = nullptr;
	x.p.out = out_dev;
	x.p.m = m;
	x.p.k = k;
	x.p.n = n;
	x.p.mult = in_scale * wt_scale / out_scale;     // tools/charsiu_matmul.c:45
	x.p.zp_out = (float)out_zp;
	x.p.zp_a = in_zp;
	x.p.zp_w = wt_zp;
	x.off_w = (uint32_t)ow;
	x.off_b = (uint32_t)ob;
	x.done_count = g->d_sync;
	x.done_flag = g->d_flag;
	x.seq = seq;
	// the smallest parameter block that holds the job (its first bytes are
	// the same in every size)
	const dim3 grid((n + 31) / 32, (m + 31) / 32);
	const size_t used = ob + sb;
	const void *fn = used <= I8_INLINE_W0 * 16 ? (const void *)i8mm_simt_inline_kernel<I8_INLINE_W0>
			 : used <= I8_INLINE_W1 * 16 ? (const void *)i8mm_simt_inline_kernel<I8_INLINE_W1>
						     : (const void *)i8mm_simt_inline_kernel<I8_INLINE_W2>;
	void *args[1] = {&x};
	if (cudaLaunchKernel(fn, grid, dim3(256), args, 0, g->stream) != cudaSuccess ||
	    cudaGetLastError() != cudaSuccess) {
		whine(g, "the int8 launch failed");
		retire(g, "a launch failed");
		return -1;
	}
	g->launches++;
	const double t1 = now_us();
	const double mb = (double)(sa + sw) / 1e6;
	if (wait_direct(g, seq, t0, mb, k))
		return -1;
	const double t2 = now_us();
	memcpy(out, g->h_i8, (size_t)m * n);
	const double t3 = now_us();
	g->calls++;
	g->weight_mb += mb;
	g->h2d_us += t1 - t0;
	g->d2h_us += t3 - t2;
	g->busy_us += t3 - t0;
	return 0;
}

extern "C" {

int charsiu_gpu_matmul_i8_flat(struct charsiu_gpu *g, unsigned m, unsigned k, unsigned n,
			       const uint8_t *a, const uint8_t *w, const int32_t *bias,
			       float in_scale, float wt_scale, float out_scale, int in_zp,
			       int wt_zp, int out_zp, int8_t *out)
{
	if (!g)
		return -1;
	g->call_no++;
	if (g->dead) {
		whine(g, "the GPU path is already retired");
		return -1;
	}
	if (!m || !k || !n || !a || !w || !bias || !out)
		return -1;
	if (injected(g, 1)) {
		whine(g, "the launch failed (injected, M=%u K=%u N=%u)", m, k, n);
		retire(g, "a launch failed");
		return -1;
	}
	cudaSetDevice(g->device);
	const size_t sa = (size_t)m * k, sw = (size_t)n * k, sb = (size_t)n * 4;
	const size_t oa = 0, ow = (sa + 15) & ~(size_t)15, ob = (ow + sw + 15) & ~(size_t)15;
	const size_t oo = (ob + sb + 15) & ~(size_t)15, total = oo + (size_t)m * n;
	if (g->direct && oo <= I8_INLINE_BYTES)
		return matmul_i8_direct(g, m, k, n, a, w, bias, in_scale, wt_scale, out_scale, in_zp,
					wt_zp, out_zp, out);
	if (!grow_dev(g->d_i8, g->cap_di8, total) || !grow_host(g->h_i8, g->cap_hi8, total)) {
		whine(g, "a staging buffer would not allocate");
		return -1;
	}
	// a direct call (the default): the kernel writes the bytes into mapped
	// host memory and its last CTA raises the sequence flag -- no read-back
	// copy and no event in the call
	int8_t *out_map = nullptr;
	if (g->direct) {
		out_map = reinterpret_cast<int8_t *>(dev_view(g->h_i8));
		if (!out_map) {
			whine(g, "a staging buffer has no device address");
			return -1;
		}
		out_map += oo;
	}
	const double t0 = now_us();
	{
		ParCopy pc;
		pc.add(g->h_i8 + oa, a, sa);
		pc.add(g->h_i8 + ow, w, sw);
		pc.add(g->h_i8 + ob, bias, sb);
		par_copy(g, pc);
	}
	cudaMemcpyAsync(g->d_i8, g->h_i8, oo, cudaMemcpyHostToDevice, g->stream);
	const double t1 = now_us();

	I8Params p = {};
	p.a = g->d_i8 + oa;
	p.w = g->d_i8 + ow;
	p.bias = reinterpret_cast<const int32_t *>(g->d_i8 + ob);
	p.out = out_map ? out_map : reinterpret_cast<int8_t *>(g->d_i8 + oo);
	uint32_t seq = 0;
	if (out_map) {
		seq = ++g->seq ? g->seq : ++g->seq;     // never 0, the flag's reset value
		p.done_count = g->d_sync;
		p.done_flag = g->d_flag;
		p.seq = seq;
	}
	p.m = m;
	p.k = k;
	p.n = n;
	p.mult = in_scale * wt_scale / out_scale;     // tools/charsiu_matmul.c:45
	p.zp_out = (float)out_zp;
	p.zp_a = in_zp;
	p.zp_w = wt_zp;
	if (!out_map)
		cudaEventRecord(g->ev_k0, g->stream);
	// M = 1 (a matvec): dp4a on the CUDA cores; M > 1: the tensor cores
	if (m == 1)
		i8mv_kernel<<<(n + I8MV_COLS - 1) / I8MV_COLS, 256, 0, g->stream>>>(p);
	else if (n <= 64)
		i8mm_tc_kernel<64><<<dim3((n + 63) / 64, (m + I8TC_M - 1) / I8TC_M), 128, 0,
				    g->stream>>>(p, g->d_err);
	else
		i8mm_tc_kernel<128><<<dim3((n + 127) / 128, (m + I8TC_M - 1) / I8TC_M), 128, 0,
				     g->stream>>>(p, g->d_err);
	if (cudaGetLastError() != cudaSuccess) {
		whine(g, "the int8 launch failed");
		retire(g, "a launch failed");
		return -1;
	}
	g->launches++;
	if (out_map) {
		const double mbd = (double)(sa + sw) / 1e6;
		if (wait_direct(g, seq, t0, mbd, k))
			return -1;
		const double t2 = now_us();
		ParCopy pc;
		pc.add(out, g->h_i8 + oo, (size_t)m * n);
		par_copy(g, pc);
		const double t3 = now_us();
		g->calls++;
		g->weight_mb += mbd;
		g->h2d_us += t1 - t0;
		g->d2h_us += t3 - t2;
		g->busy_us += t3 - t0;
		return 0;
	}
	cudaEventRecord(g->ev_k1, g->stream);
	cudaMemcpyAsync(g->h_i8 + oo, g->d_i8 + oo, (size_t)m * n, cudaMemcpyDeviceToHost,
			g->stream);
	cudaEventRecord(g->ev_done, g->stream);
	const double mb = (double)(sa + sw) / 1e6;
	if (finish(g, t0, mb, k, n))
		return -1;
	const double t2 = now_us();
	memcpy(out, g->h_i8 + oo, (size_t)m * n);
	float kms = 0;
	if (cudaEventElapsedTime(&kms, g->ev_k0, g->ev_k1) != cudaSuccess) {
		kms = 0;
		cudaGetLastError();
	}
	const double t3 = now_us();
	g->calls++;
	g->weight_mb += mb;
	g->h2d_us += t1 - t0;
	g->kern_ms += kms;
	g->d2h_us += t3 - t2;
	g->busy_us += t3 - t0;
	return 0;
}

int charsiu_gpu_matmul_i8(struct charsiu_gpu *g, const struct charsiu_job *job,
			  const uint8_t *a, const uint8_t *w, const int32_t *bias, int8_t *out)
{
	if (!g || !job)
		return -1;
	const RefJob *j = reinterpret_cast<const RefJob *>(job);
	if (j->mm.wdtype != REF_INT8 || j->mm.adtype != REF_INT8) {
		whine(g, "only int8 weights and activations (wdtype %d adtype %d)", j->mm.wdtype,
		      j->mm.adtype);
		return -1;
	}
	if (j->acc_out) {
		whine(g, "acc_out jobs return the raw accumulator; use the matvec path");
		return -1;
	}
	return charsiu_gpu_matmul_i8_flat(g, j->mm.m, j->mm.k, j->mm.n, a, w, bias, j->input_scale,
					  j->weight_scale, j->output_scale, j->input_zero_point,
					  j->weight_zero_point, j->output_zero_point, out);
}

unsigned long charsiu_gpu_calls(const struct charsiu_gpu *g)
{
	return g ? g->calls : 0;
}

unsigned long charsiu_gpu_launches(const struct charsiu_gpu *g)
{
	return g ? g->launches : 0;
}

const char *charsiu_gpu_error(const struct charsiu_gpu *g)
{
	return g ? g->err.c_str() : "no layer";
}

int charsiu_gpu_dead(const struct charsiu_gpu *g)
{
	return g ? g->dead : 1;
}

// What the device actually did, printed whether it went well or not
// (src/npudev.c:264-295).
// Internal to the library (host/llama_gpu.c): the decode loop lends the
// layer its pool for the large copies, so that two sets of spinning host
// threads never compete for the cores; NULL takes it back (single-threaded
// copies from then on). The layer never frees a lent pool.
void charsiu_gpu_lend_pool(struct charsiu_gpu *g, struct pool *p)
{
	if (!g)
		return;
	if (g->copy_pool_owned)
		pool_free(g->copy_pool);
	g->copy_pool = p;
	g->copy_pool_owned = false;
	g->copy_pool_tried = true;
}

void charsiu_gpu_report(const struct charsiu_gpu *g)
{
	if (!g)
		return;
	double mbs = 0;
	for (const Ent &e : g->ent)
		mbs += e.weight_mb;
	fprintf(stderr, "charsiu GPU: device %d (rank %u of %u), %zu tensors (%.1f MB), "
			"%lu calls, %lu launches, %.2f MB per call%s\n",
		g->device, g->rank, g->world, g->ent.size(), mbs, g->calls, g->launches,
		g->calls ? g->weight_mb / (double)g->calls : 0.0,
		g->dead ? "  (RETIRED: it stopped answering)" : "");
	if (g->calls)
		fprintf(stderr,
			"charsiu GPU: %.1f ms in the device path, %.2f GB/s of weights, %.1f us a "
			"call\ncharsiu GPU: of that, %.1f ms copying in, %.2f ms in kernels, "
			"%.1f ms reading back\n",
			g->busy_us / 1e3, g->weight_mb / g->busy_us * 1e3,
			g->busy_us / (double)g->calls, g->h2d_us / 1e3, g->kern_ms,
			g->d2h_us / 1e3);
	else
		fprintf(stderr, "charsiu GPU: NOTHING RAN ON THE GPU. Every number in this run "
				"came from the CPU.\n");
}

int charsiu_gpu_block_dots(struct charsiu_gpu *g, int id, const int8_t *q, int32_t *dots)
{
	if (!g || g->dead || !q || !dots || id < 0 || (size_t)id >= g->ent.size())
		return -1;
	cudaSetDevice(g->device);
	const Ent &e = g->ent[id];
	if (e.type == TYPE_Q6_K) {
		whine(g, "block dots are of 32-element blocks: q8_0 and q4_0 only (%s)", e.name);
		return -1;
	}
	const size_t cnt = (size_t)e.rows * e.nb;
	if (!grow_dev(g->d_q, g->cap_dq, (size_t)e.nb * 32) ||
	    !grow_dev(g->d_dots, g->cap_dots, cnt ? cnt : 1))
		return -1;
	if (cudaMemcpy(g->d_q, q, (size_t)e.nb * 32, cudaMemcpyHostToDevice) != cudaSuccess)
		return -1;
	if (cnt) {
		block_dots_kernel<<<(unsigned)((cnt + 255) / 256), 256, 0, g->stream>>>(
			e.data, e.type, (uint32_t)e.rows, e.nb, g->d_q, g->d_dots);
		g->launches++;
	}
	if (cudaStreamSynchronize(g->stream) != cudaSuccess ||
	    cudaMemcpy(dots, g->d_dots, cnt * sizeof(int32_t), cudaMemcpyDeviceToHost) !=
		    cudaSuccess)
		return -1;
	return 0;
}

int charsiu_gpu_inject(struct charsiu_gpu *g, unsigned long at, unsigned long count, int kind)
{
	if (!g || kind < 0 || kind > 3)
		return -1;
	g->inj_at = at;
	g->inj_count = count;
	g->inj_kind = count ? kind : 0;
	return 0;
}

} // extern "C"
