// SPDX-License-Identifier: GPL-2.0-or-later
// charsiu's NPU device layer (include/charsiu_llm.h:186-200, src/npudev.c)
// over CUDA: the host side of include/charsiu_npu.h.
//
// npudev.c slices each projection into hardware jobs, submits them, waits
// for the fence and forms y = (float)acc * d1 * scale from the raw int32
// accumulators. Here a projection (or a group of them) is one launch of
// npumv_kernel, which forms the same y on the GPU: the activation travels in
// the launch's own parameters, y lands in mapped pinned host memory, and the
// last CTA raises a sequence flag the host spins on -- no copy engine, graph
// or event in the call. The conventions are npudev.c's: whine once, a budget
// of CHARSIU_GPU_SLOW_US plus a millisecond a megabyte, three slow calls in a
// row retire the layer, and a report that says so when nothing ran.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <new>
#include <string>
#include <vector>

#include "charsiu_npu.h"

#include "host_copy.h"
#include "npu_internal.h"
#include "npumv.cuh"
#include "ref_abi.h"

using namespace cgpu;

namespace {

double now_us()
{
	timespec t;
	clock_gettime(CLOCK_MONOTONIC, &t);
	return (double)t.tv_sec * 1e6 + (double)t.tv_nsec / 1e3;
}

struct NpuEnt {
	const void *key;          // the caller's npu_tensor
	char name[80];
	uint64_t n, k;
	uint32_t kp;              // padded row bytes
	int8_t *w;                // [n][kp] (device)
	float *scale;             // [n] (device)
	double weight_mb;
};

} // namespace

struct charsiu_npu {
	int device = 0;
	int sm_count = 0;
	unsigned max_k = 0, max_n = 0, max_tensors = 0;
	cudaStream_t stream = nullptr;
	std::vector<NpuEnt> ent;
	float *h_y = nullptr;              // mapped pinned: every y of a call
	size_t cap_y = 0;
	uint32_t *d_count = nullptr;       // CTAs done (device)
	unsigned long long *d_tstart = nullptr;
	volatile uint32_t *h_flag = nullptr;
	uint32_t *d_flag = nullptr;
	uint32_t seq = 0;
	NpuInline<NPU_INLINE_WORDS> *inl = nullptr;
	bool smem_set[12] = {};
	int occ[12] = {};                  // CTAs an SM of each kernel form, asked once
	unsigned long calls = 0, launches = 0;
	double busy_us = 0, kern_ms = 0, weight_mb = 0, slow_us = 100000;
	int strikes = 0, dead = 0, whined = 0, no_pdl = 0;
	std::string err;
	struct pool *pool = nullptr;       // lent by the decode loop for large read-backs
};

namespace {

void whine(charsiu_npu *g, const char *fmt, ...)
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

void retire(charsiu_npu *g, const char *why)
{
	if (g->dead)
		return;
	g->dead = 1;
	g->strikes = 3;
	fprintf(stderr, "charsiu: the GPU stopped answering (%s); everything from here runs on "
			"the CPU\n", why);
}

int check_group(charsiu_npu *g, const int *ids, unsigned n, uint64_t k)
{
	if (!ids || !n || n > (unsigned)NPU_MAX_TENSORS)
		return -1;
	for (unsigned i = 0; i < n; i++) {
		if (ids[i] < 0 || (size_t)ids[i] >= g->ent.size())
			return -1;
		if (g->ent[ids[i]].k != k) {
			whine(g, "the activation is not this tensor's K (K=%llu N=%llu)",
			      (unsigned long long)k, (unsigned long long)g->ent[ids[i]].n);
			return -1;
		}
	}
	return 0;
}

void fill(charsiu_npu *g, NpuParams &p, const int *ids, unsigned n, float *const *ys, float d1,
	  const int8_t *q1, const float *d1p = nullptr)
{
	memset(&p, 0, sizeof(p));
	uint32_t acc = 0;
	for (unsigned i = 0; i < n; i++) {
		const NpuEnt &e = g->ent[ids[i]];
		p.t[i].w = e.w;
		p.t[i].scale = e.scale;
		p.t[i].y = ys[i];
		p.t[i].rows = (uint32_t)e.n;
		acc += (uint32_t)e.n;
		p.t[i].row_end = acc;
	}
	p.ntensor = n;
	p.total_rows = acc;
	p.kp = g->ent[ids[0]].kp;
	p.d1 = d1;
	p.d1p = d1p;
	p.q1 = q1;
}

// One launch: the inline form when `inl` (its .p is p), else q1 from p.q1.
// npumv_kernel<W, U>: W warps split K, U chunks a lane a row a pass -- K up
// to 2048 four warps (eight CTAs an SM), 4096 eight, 8192 sixteen, past that
// sixteen with two chunks a lane. (At K = 8192 eight warps with two chunks a
// lane measured 4.7-4.8 against 4.4-4.7 us.)
int launch(charsiu_npu *g, const NpuParams &p, const void *inl, cudaStream_t st)
{
#define NPU_FNS(W, U) \
	{(const void *)npumv_kernel<W, U>, (const void *)npumv_inline_kernel<W, U, 128>, \
	 (const void *)npumv_inline_kernel<W, U, NPU_INLINE_WORDS>}
	static const void *const fns[4][3] = {NPU_FNS(4, 1), NPU_FNS(8, 1), NPU_FNS(16, 1),
					      NPU_FNS(16, 2)};
#undef NPU_FNS
	static const int warps[4] = {4, 8, 16, 16};
	const uint32_t nch = p.kp / 16;
	const int si = nch <= 128 ? 0 : nch <= 256 ? 1 : nch <= 512 ? 2 : 3;
	const int form = inl ? (p.kp <= 128 * 16 ? 1 : 2) : 0;
	const void *fn = fns[si][form];
	const int slot = si * 3 + form;
	const int threads = warps[si] * 32;
	const size_t smem = npumv_smem_bytes(p.kp, warps[si]);
	if (smem > NPU_SMEM_MAX)
		return -1;
	if (!g->smem_set[slot]) {
		if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
					 (int)NPU_SMEM_MAX) != cudaSuccess)
			return -1;
		g->smem_set[slot] = true;
	}
	if (!g->occ[slot]) {
		int occ = 0;
		if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, threads, NPU_SMEM_MAX) !=
			    cudaSuccess || occ < 1)
			return -1;
		g->occ[slot] = occ;
	}
	const uint32_t groups = (p.total_rows + NPU_GROUP_ROWS - 1) / NPU_GROUP_ROWS;
	unsigned grid = (unsigned)g->occ[slot] * g->sm_count;
	if (groups < grid)
		grid = groups ? groups : 1;
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
	void *args[1] = {inl ? const_cast<void *>(inl) : const_cast<NpuParams *>(&p)};
	if (cudaLaunchKernelExC(&cfg, fn, args) != cudaSuccess)
		return -1;
	g->launches++;
	return 0;
}

// The host call: q1 (k bytes, zero-padded to kp by the copy) and d1 in, every
// ys[i] out, one launch and a flag.
int run(charsiu_npu *g, const int *ids, unsigned n, const int8_t *q1, float d1, uint64_t k,
	float **ys)
{
	if (g->dead) {
		whine(g, "the GPU path is already retired");
		return -1;
	}
	if (!q1 || !ys || check_group(g, ids, n, k))
		return -1;
	cudaSetDevice(g->device);
	size_t ytot = 0;
	double mb = 0;
	for (unsigned i = 0; i < n; i++) {
		ytot += g->ent[ids[i]].n;
		mb += g->ent[ids[i]].weight_mb;
	}
	if (ytot > g->cap_y) {
		whine(g, "more outputs than the layer was opened for");
		return -1;
	}
	float *y_dev = nullptr;
	if (cudaHostGetDevicePointer((void **)&y_dev, g->h_y, 0) != cudaSuccess) {
		whine(g, "a staging buffer has no device address");
		return -1;
	}
	const double t0 = now_us();
	float *yd[NPU_MAX_TENSORS];
	size_t off = 0;
	for (unsigned i = 0; i < n; i++) {
		yd[i] = y_dev + off;
		off += g->ent[ids[i]].n;
	}
	const uint32_t seq = ++g->seq ? g->seq : ++g->seq;     // never 0, the flag's reset value
	NpuInline<NPU_INLINE_WORDS> &a = *g->inl;
	fill(g, a.p, ids, n, yd, d1, nullptr);
	a.p.done_count = g->d_count;
	a.p.done_flag = g->d_flag;
	a.p.t_start = g->d_tstart;
	a.p.seq = seq;
	const uint32_t kp = a.p.kp;
	uint8_t *words = reinterpret_cast<uint8_t *>(a.act);
	memcpy(words, q1, k);
	memset(words + k, 0, kp - k);
	if (launch(g, a.p, &a, g->stream)) {
		whine(g, "the launch failed: %s", cudaGetErrorString(cudaGetLastError()));
		retire(g, "a launch failed");
		return -1;
	}
	// npudev.c's budget (src/npudev.c:560-573)
	const double budget = g->slow_us + mb * 1000.0;
	for (uint64_t spins = 1; g->h_flag[0] != seq; spins++) {
		if (spins & 1023)
			continue;
		const double el = now_us() - t0;
		if (el <= budget)
			continue;
		const cudaError_t e = cudaStreamQuery(g->stream);
		if (e != cudaSuccess && e != cudaErrorNotReady) {
			whine(g, "CUDA error %s", cudaGetErrorString(e));
			retire(g, "a CUDA error");
			return -1;
		}
		if (e == cudaSuccess && g->h_flag[0] != seq) {
			whine(g, "a call finished without signalling");
			retire(g, "a call finished without signalling");
			return -1;
		}
		if (el > budget + 10e6) {
			whine(g, "a call did not finish");
			retire(g, "it stopped answering");
			return -1;
		}
	}
	std::atomic_thread_fence(std::memory_order_acquire);
	const double took = now_us() - t0;
	if (took > budget) {
		if (++g->strikes >= 3) {
			whine(g, "three slow calls in a row");
			retire(g, "it stopped answering in time");
			return -1;
		}
	} else {
		g->strikes = 0;
	}
	{
		// the outputs out of mapped memory, on the lent threads when large
		ParCopy pc;
		off = 0;
		for (unsigned i = 0; i < n; i++) {
			const size_t cnt = g->ent[ids[i]].n;
			pc.add(ys[i], g->h_y + off, cnt * sizeof(float));
			off += cnt;
		}
		pc.run(g->pool);
	}
	g->calls++;
	g->weight_mb += mb;
	g->kern_ms += g->h_flag[1] * 1e-6;
	g->busy_us += now_us() - t0;
	return 0;
}

} // namespace

// ---- what the decode step asks of the layer --------------------------------

namespace cgpu {

int npu_layer_device(const charsiu_npu *g)
{
	return g->device;
}

bool npu_layer_dead(const charsiu_npu *g)
{
	return g->dead != 0;
}

bool npu_layer_tensor(const charsiu_npu *g, int id, uint64_t *k, uint64_t *n, uint32_t *kp)
{
	if (id < 0 || (size_t)id >= g->ent.size())
		return false;
	*k = g->ent[id].k;
	*n = g->ent[id].n;
	*kp = g->ent[id].kp;
	return true;
}

int npu_layer_matvec_dev_d1(charsiu_npu *g, const int *ids, unsigned n, const int8_t *q1,
			    const float *d1, float *const *ys, cudaStream_t st)
{
	if (g->dead || !q1 || !d1 || !ys || ((uintptr_t)q1 & 15) || !ids || !n ||
	    n > (unsigned)NPU_MAX_TENSORS || ids[0] < 0 || (size_t)ids[0] >= g->ent.size() ||
	    check_group(g, ids, n, g->ent[ids[0]].k))
		return -1;
	NpuParams p;
	fill(g, p, ids, n, ys, 0.0f, q1, d1);
	return launch(g, p, nullptr, st);
}

unsigned long npu_layer_launches(const charsiu_npu *g)
{
	return g->launches;
}

} // namespace cgpu

extern "C" {

struct charsiu_npu *charsiu_npu_open(unsigned max_k, unsigned max_n, unsigned max_tensors)
{
	const char *e = getenv("CHARSIU_GPU_DEVICE");
	return charsiu_npu_open_ex(max_k, max_n, max_tensors, e ? atoi(e) : 0);
}

struct charsiu_npu *charsiu_npu_open_ex(unsigned max_k, unsigned max_n, unsigned max_tensors,
					int device)
{
	int ndev = 0;
	if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
		fprintf(stderr, "charsiu: no CUDA device %d\n", device);
		return nullptr;
	}
	if (!max_k || max_k > (unsigned)NPU_INLINE_WORDS * 16 || !max_n || !max_tensors)
		return nullptr;
	cudaDeviceProp prop;
	if (cudaSetDevice(device) != cudaSuccess ||
	    cudaGetDeviceProperties(&prop, device) != cudaSuccess)
		return nullptr;
	if (prop.major != 10 || prop.minor != 0) {
		fprintf(stderr, "charsiu: device %d is sm_%d%d; this build is sm_100a only\n", device,
			prop.major, prop.minor);
		return nullptr;
	}
	charsiu_npu *g = new (std::nothrow) charsiu_npu;
	if (!g)
		return nullptr;
	g->device = device;
	g->sm_count = prop.multiProcessorCount;
	g->max_k = max_k;
	g->max_n = max_n;
	g->max_tensors = max_tensors;
	if (const char *e = getenv("CHARSIU_GPU_SLOW_US"))
		g->slow_us = (double)strtoul(e, nullptr, 0);
	g->no_pdl = getenv("CHARSIU_GPU_NO_PDL") != nullptr;
	g->ent.reserve(max_tensors);
	g->cap_y = (size_t)max_n * NPU_MAX_TENSORS;
	g->inl = new (std::nothrow) NpuInline<NPU_INLINE_WORDS>();
	bool ok = g->inl != nullptr;
	ok = ok && cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking) == cudaSuccess;
	ok = ok && cudaHostAlloc((void **)&g->h_y, g->cap_y * sizeof(float), cudaHostAllocMapped) ==
			   cudaSuccess;
	ok = ok && cudaHostAlloc((void **)&g->h_flag, 4 * sizeof(uint32_t), cudaHostAllocMapped) ==
			   cudaSuccess;
	ok = ok && cudaHostGetDevicePointer((void **)&g->d_flag, (void *)g->h_flag, 0) == cudaSuccess;
	ok = ok && cudaMalloc((void **)&g->d_count, sizeof(uint32_t)) == cudaSuccess;
	ok = ok && cudaMemset(g->d_count, 0, sizeof(uint32_t)) == cudaSuccess;
	ok = ok && cudaMalloc((void **)&g->d_tstart, sizeof(unsigned long long)) == cudaSuccess;
	if (!ok) {
		charsiu_npu_close(g);
		return nullptr;
	}
	for (int i = 0; i < 4; i++)
		g->h_flag[i] = 0;
	return g;
}

static_assert(NPU_MAX_TENSORS <= ParCopy::MAX_SEG, "a launch group's outputs in one copy");

// Internal to the library (host/llama_gpu.c): the decode loop lends its host
// threads for the large read-backs; NULL takes them back. Never freed here.
void charsiu_npu_lend_pool(struct charsiu_npu *g, struct pool *p)
{
	if (g)
		g->pool = p;
}

void charsiu_npu_close(struct charsiu_npu *g)
{
	if (!g)
		return;
	cudaSetDevice(g->device);
	if (g->stream)
		cudaStreamSynchronize(g->stream);
	for (NpuEnt &e : g->ent) {
		cudaFree(e.w);
		cudaFree(e.scale);
	}
	if (g->h_y)
		cudaFreeHost(g->h_y);
	if (g->h_flag)
		cudaFreeHost((void *)g->h_flag);
	if (g->d_count)
		cudaFree(g->d_count);
	if (g->d_tstart)
		cudaFree(g->d_tstart);
	if (g->stream)
		cudaStreamDestroy(g->stream);
	delete g->inl;
	delete g;
}

int charsiu_npu_add_flat(struct charsiu_npu *g, const int8_t *q, const float *scale, uint64_t n,
			 uint64_t k, const char *name)
{
	if (!g || !q || !scale || !n || !k)
		return -1;
	if (g->dead) {
		whine(g, "the GPU path is already retired");
		return -1;
	}
	if (g->ent.size() >= g->max_tensors) {
		whine(g, "no tensor slots left (K=%llu N=%llu)", (unsigned long long)k,
		      (unsigned long long)n);
		return -1;
	}
	if (n > g->max_n || k > g->max_k) {
		whine(g, "wider than the layer was opened for (K=%llu N=%llu)",
		      (unsigned long long)k, (unsigned long long)n);
		return -1;
	}
	cudaSetDevice(g->device);
	NpuEnt e = {};
	snprintf(e.name, sizeof(e.name), "%s", name ? name : "");
	e.n = n;
	e.k = k;
	e.kp = (uint32_t)((k + 15) & ~(uint64_t)15);
	e.weight_mb = (double)n * (double)k / 1e6;
	bool ok = cudaMalloc((void **)&e.w, (size_t)n * e.kp) == cudaSuccess;
	ok = ok && cudaMalloc((void **)&e.scale, (size_t)n * sizeof(float)) == cudaSuccess;
	ok = ok && cudaMemset(e.w, 0, (size_t)n * e.kp) == cudaSuccess;
	ok = ok && cudaMemcpy2D(e.w, e.kp, q, k, k, n, cudaMemcpyHostToDevice) == cudaSuccess;
	ok = ok && cudaMemcpy(e.scale, scale, (size_t)n * sizeof(float), cudaMemcpyHostToDevice) ==
			   cudaSuccess;
	if (!ok) {
		cudaFree(e.w);
		cudaFree(e.scale);
		whine(g, "a device buffer would not allocate (K=%llu N=%llu)", (unsigned long long)k,
		      (unsigned long long)n);
		return -1;
	}
	g->ent.push_back(e);
	return (int)g->ent.size() - 1;
}

int charsiu_npu_add(struct charsiu_npu *g, const struct npu_tensor *t)
{
	if (!g || !t)
		return -1;
	const RefNpuTensor *nt = reinterpret_cast<const RefNpuTensor *>(t);
	for (size_t i = 0; i < g->ent.size(); i++)
		if (g->ent[i].key == t)
			return (int)i;
	if (nt->kgroup && nt->kgroup != nt->k) {
		whine(g, "%s has a scale every %llu of K; the device arithmetic takes one a row",
		      nt->name, (unsigned long long)nt->kgroup);
		return -1;
	}
	if (nt->kscale) {
		whine(g, "%s carries a k factor, which the device arithmetic does not apply",
		      nt->name);
		return -1;
	}
	const int id = charsiu_npu_add_flat(g, nt->q, nt->scale, nt->n, nt->k, nt->name);
	if (id >= 0)
		g->ent[id].key = t;
	return id;
}

int charsiu_npu_matvec_flat(struct charsiu_npu *g, const int *ids, unsigned n, const int8_t *q1,
			    float d1, unsigned k, float **ys)
{
	if (!g)
		return -1;
	return run(g, ids, n, q1, d1, k, ys);
}

int charsiu_npu_matvec(struct charsiu_npu *g, int id, const struct charsiu_act *a, float *y)
{
	if (!g || !a || !y)
		return -1;
	const RefAct *ra = reinterpret_cast<const RefAct *>(a);
	float *ys[1] = {y};
	return run(g, &id, 1, ra->q1, ra->d1, (uint64_t)ra->n, ys);
}

int charsiu_npu_matvec_group(struct charsiu_npu *g, const int *ids, unsigned n,
			     const struct charsiu_act *a, float **ys)
{
	if (!g || !a || !ys)
		return -1;
	const RefAct *ra = reinterpret_cast<const RefAct *>(a);
	return run(g, ids, n, ra->q1, ra->d1, (uint64_t)ra->n, ys);
}

int charsiu_npu_matvec_dev(struct charsiu_npu *g, const int *ids, unsigned n, const int8_t *q1,
			   float d1, float *const *ys, void *stream)
{
	if (!g || g->dead || !q1 || !ys || ((uintptr_t)q1 & 15) || !ids || !n ||
	    n > (unsigned)NPU_MAX_TENSORS || ids[0] < 0 || (size_t)ids[0] >= g->ent.size() ||
	    check_group(g, ids, n, g->ent[ids[0]].k))
		return -1;
	cudaSetDevice(g->device);
	NpuParams p;
	fill(g, p, ids, n, ys, d1, q1);
	return launch(g, p, nullptr, stream ? (cudaStream_t)stream : g->stream);
}

unsigned long charsiu_npu_submits(const struct charsiu_npu *g)
{
	return g ? g->calls : 0;
}

void charsiu_npu_report(const struct charsiu_npu *g)
{
	if (!g)
		return;
	fprintf(stderr, "charsiu NPU format on the GPU: %zu tensors, %lu calls, %lu launches, "
			"%.2f MB per call%s\n",
		g->ent.size(), g->calls, g->launches,
		g->calls ? g->weight_mb / (double)g->calls : 0.0,
		g->dead ? "  (RETIRED: it stopped answering)" : "");
	if (g->calls)
		fprintf(stderr, "charsiu NPU format on the GPU: %.1f ms in calls, %.2f GB/s of "
				"weights a call, %.1f us a call (%.1f us in the kernels)\n",
			g->busy_us / 1e3, g->weight_mb / g->busy_us * 1e3,
			g->busy_us / (double)g->calls, g->kern_ms * 1e3 / (double)g->calls);
	else
		fprintf(stderr, "charsiu NPU format on the GPU: NOTHING RAN ON THE GPU. Every "
				"number in this run came from the CPU.\n");
}

const char *charsiu_npu_error(const struct charsiu_npu *g)
{
	return g ? g->err.c_str() : "";
}

int charsiu_npu_dead(const struct charsiu_npu *g)
{
	return g ? g->dead : 1;
}

} // extern "C"
