// SPDX-License-Identifier: GPL-2.0-or-later
// Inline-PTX helpers for sm_100a: mbarriers, the untiled bulk copy engine
// (global -> this CTA's shared memory, one destination), programmatic
// dependent launch, and the mixed-sign dp4a.
#pragma once

#include <cstdint>

namespace cgpu {

// every bounded wait in this library gives up after this long
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;   // one second

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
	return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
	asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;"
		     :: "r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
	asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// One arrival that also tells the barrier how many bytes the copy will land.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
	asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
		     :: "r"(smem_addr(bar)), "r"(bytes) : "memory");
}

// A plain arrival (release semantics at CTA scope).
__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
	asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];"
		     :: "r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
	uint32_t ok;
	asm volatile("{\n\t.reg .pred p;\n\t"
		     "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
		     "selp.u32 %0, 1, 0, p;\n\t}"
		     : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
	return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns()
{
	uint64_t t;
	asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
	return t;
}

// Wait for phase `parity` of `bar`, for at most `limit_ns`. false: gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
						  uint64_t limit_ns)
{
	if (mbar_try_wait(bar, parity))
		return true;
	uint64_t t0 = globaltimer_ns();
	while (!mbar_try_wait(bar, parity))
		if (globaltimer_ns() - t0 > limit_ns)
			return false;
	return true;
}

// Untiled bulk copy, global -> shared memory of this CTA, completing `bytes`
// of transaction count on `bar`. dst and src 16-byte aligned, bytes a
// multiple of 16. Every bulk copy in this library has this one destination.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
					 uint64_t *bar)
{
	asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
		     " [%0], [%1], %2, [%3];"
		     :: "r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
		     : "memory");
}

// Tiled tensor copies, global -> shared memory of this CTA, through the tensor
// map at generic address `map` (a __grid_constant__ kernel parameter): the
// box at coordinates (x, y[, z]) lands densely, x fastest, and completes the
// whole box's bytes on `bar` (out-of-range elements read as zero). x times
// the element size must be a multiple of 16 bytes; no cluster multicast.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *map, int x, int y,
					    uint64_t *bar)
{
	asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
		     " [%0], [%1, {%2, %3}], [%4];"
		     :: "r"(smem_addr(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
		     : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const void *map, int x, int y, int z,
					    uint64_t *bar)
{
	asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
		     " [%0], [%1, {%2, %3, %4}], [%5];"
		     :: "r"(smem_addr(dst)), "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
		     : "memory");
}

// Order this thread's earlier generic-proxy accesses to shared memory before
// later async-proxy (bulk copy) writes to it.
__device__ __forceinline__ void fence_proxy_async_smem()
{
	asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Programmatic dependent launch: block until the grid this one depends on
// has completed and its writes are visible; let the next grid start launching.
__device__ __forceinline__ void pdl_wait()
{
	asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void pdl_launch_dependents()
{
	asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// barrier `id` (1..15) over `threads` threads of the CTA
__device__ __forceinline__ void named_barrier(int id, int threads)
{
	asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(threads) : "memory");
}

// atomic add at device scope with acquire-release ordering; returns the old value
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t *addr, uint32_t v)
{
	uint32_t old;
	asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;"
		     : "=r"(old) : "l"(addr), "r"(v) : "memory");
	return old;
}

// The arrival words other GPUs write over NVLink (the matvecs fused with
// their all-gather): a system-scope acquire load on the waiting side; on the
// signalling side a system-scope acq_rel fence and relaxed system-scope adds
// after it, which together release everything ordered before the fence.
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p)
{
	uint32_t v;
	asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
	return v;
}

__device__ __forceinline__ void fence_acq_rel_sys()
{
	asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__device__ __forceinline__ void red_relaxed_sys_add(uint32_t *p, uint32_t v)
{
	asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

// sum of four (unsigned byte of a) * (signed byte of b), plus c
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c)
{
	int d;
	asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
	return d;
}

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c)
{
	return __dp4a(static_cast<int>(a), static_cast<int>(b), c);
}

// Packed fp32 pairs (sm_100), held as one 64-bit register (low word = first
// lane), so no packing moves sit between consecutive operations. Each lane
// rounds to nearest as mul.rn.f32 / add.rn.f32 / fma.rn.f32 do.
//
// Unlike the scalar forms, a mul.rn.f32x2 whose result feeds an
// add.rn.f32x2 is contracted by the assembler into one fused multiply-add
// (seen on sm_100a with CUDA 12.9: 1-ulp differences), so code that needs
// the product rounded before the sum uses fma2_rn(product, 1.0, s) with the
// 1.0 in a register the assembler cannot see into (a kernel parameter):
// that rounds once, after the exact product-times-one, which is the add.
__device__ __forceinline__ uint64_t pack2(float lo, float hi)
{
	return (uint64_t)__float_as_uint(hi) << 32 | __float_as_uint(lo);
}

__device__ __forceinline__ uint64_t pack2u(uint32_t lo, uint32_t hi)
{
	return (uint64_t)hi << 32 | lo;
}

__device__ __forceinline__ float lo2(uint64_t v)
{
	return __uint_as_float((uint32_t)v);
}

__device__ __forceinline__ float hi2(uint64_t v)
{
	return __uint_as_float((uint32_t)(v >> 32));
}

__device__ __forceinline__ uint64_t mul2_rn(uint64_t a, uint64_t b)
{
	uint64_t d;
	asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
	return d;
}

__device__ __forceinline__ uint64_t add2_rn(uint64_t a, uint64_t b)
{
	uint64_t d;
	asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
	return d;
}

__device__ __forceinline__ uint64_t fma2_rn(uint64_t a, uint64_t b, uint64_t c)
{
	uint64_t d;
	asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
	return d;
}

// 16 bytes (2 bytes) of streamed read-only data: no L1 allocation
__device__ __forceinline__ uint4 ldg_stream(const uint8_t *p)
{
	uint4 v;
	asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
		     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
	return v;
}

__device__ __forceinline__ uint16_t ldg_stream_u16(const uint8_t *p)
{
	uint16_t v;
	asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
	return v;
}

// fp16 bits -> fp32, exact for every finite value (subnormals included)
__device__ __forceinline__ float half_bits_to_float(uint16_t h)
{
	float f;
	asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
	return f;
}

} // namespace cgpu
