// Shared device helpers for the sm_100a TriMul kernels: mbarriers with bounded
// waits, TMA (cp.async.bulk.tensor) loads, tcgen05 MMA / TMEM access and the
// shared-memory matrix descriptors they consume.
//
// Every spin in these kernels is bounded: a wait that runs past FTM_WAIT_NS
// records an error code in a device word (first writer wins) and returns false,
// and the calling role then leaves its loop, drains what it issued and exits.
// Nothing here traps.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef FTM_WAIT_NS
#define FTM_WAIT_NS 2000000000ull  // 2 s: no legal wait in these kernels comes close
#endif

namespace ftm {

// ---------------------------------------------------------------- error codes
// device error word: 0 = fine; otherwise (kernel << 8) | (role << 4) | site
enum : int { KERNEL_INPUT = 1, KERNEL_CONTRACT = 2, KERNEL_OUTPUT = 3 };
enum : int { ROLE_PRODUCER = 1, ROLE_MMA = 2, ROLE_TRANSFORM = 3, ROLE_EPILOGUE = 4 };

__device__ __forceinline__ int err_code(int kernel, int role, int site) {
  return (kernel << 8) | (role << 4) | site;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------ mbarriers
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// try_wait with a suspend-time hint: the waiting thread sleeps in hardware until the
// phase completes or ~`ns` nanoseconds pass, instead of spinning on issue slots
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return done != 0;
}

// Wait for the phase of `bar` with parity `parity` to complete. Returns false
// (after recording `code` in *err) if it did not within FTM_WAIT_NS, or if
// another thread of the grid has already recorded an error. Between checks of the
// error word and the clock the thread sleeps in try_wait (up to 20 us per call).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (*reinterpret_cast<volatile int*>(err) != 0) return false;
    if (globaltimer_ns() - t0 > FTM_WAIT_NS) {
      atomicCAS(err, 0, code);
      return false;
    }
  }
}

// Drain wait used after a failure: waits (bounded) for copies / MMAs this thread
// issued to land, without looking at the error word.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait_sleep(bar, parity, 20000u)) {
    if (globaltimer_ns() - t0 > FTM_WAIT_NS) return false;
  }
  return true;
}

// Warp-uniform wait for roles that go on to issue .sync.aligned instructions:
// every lane polls, and the warp proceeds only if all lanes saw the phase.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int* err, int code) {
  const bool ok = mbar_wait(bar, parity, err, code);
  return __all_sync(0xffffffffu, ok);
}

// Programmatic dependent launch. A kernel launched with programmatic stream
// serialisation may start while its predecessor on the stream is still finishing; it
// must not touch global memory (other than prefetching tensor-map descriptors) before
// grid_dep_wait(), which returns once the predecessor grid has completed and its writes
// are visible. Each kernel releases its own dependents only after that wait, so a
// kernel can never overlap anything but the tail of its immediate predecessor.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_release() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ bool grid_failed(const int* err) {
  return *reinterpret_cast<const volatile int*>(err) != 0;
}

// ----------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// L2 prefetch of a tensor tile (no shared memory, no barrier): starts the HBM read of a
// tile the producer will load a few iterations later, so more bytes are in flight per SM
// than the shared-memory ring alone allows
__device__ __forceinline__ void tma_prefetch_l2_4d(const CUtensorMap* map, int c0, int c1, int c2,
                                                   int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(map),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// TMA tensor stores (shared -> global), bulk-group completion
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1,
                                             int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(map),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until the source shared memory of all committed stores has been read
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// wait until all committed stores are complete (globally visible)
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// generic-proxy shared-memory writes -> visible to the async proxy (UMMA, TMA)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_barrier_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, fp16/bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// arrive on `bar` once every tcgen05 op issued so far by this thread completes
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// two 32-column TMEM loads completed by one wait
__device__ __forceinline__ void tmem_ld32x2(uint32_t taddr0, uint32_t taddr1, float (&v0)[32],
                                            float (&v1)[32]);

// 32 TMEM lanes x 32 consecutive fp32 columns -> 32 registers per thread
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

#define FTM_TMEM_LD32_NOWAIT(taddr, r)                                                          \
  asm volatile(                                                                                \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "                                                \
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"                                \
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"               \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),    \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),             \
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),          \
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),          \
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),          \
        "=r"(r[31])                                                                            \
      : "r"(taddr))

__device__ __forceinline__ void tmem_ld32x2(uint32_t taddr0, uint32_t taddr1, float (&v0)[32],
                                            float (&v1)[32]) {
  uint32_t a[32], b[32];
  FTM_TMEM_LD32_NOWAIT(taddr0, a);
  FTM_TMEM_LD32_NOWAIT(taddr1, b);
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v0[i] = __uint_as_float(a[i]);
    v1[i] = __uint_as_float(b[i]);
  }
}

// 32 TMEM lanes x 16 columns, issued without waiting (pair with tmem_wait_ld)
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// 32 TMEM lanes x 8 columns, issued without waiting (pair with tmem_wait_ld)
__device__ __forceinline__ void tmem_ld8_nowait(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------- UMMA descriptors
// Shared-memory matrix descriptor (tcgen05 format, version 1) for a
// 128-byte-swizzled tile. K-major: rows of 128 B, 8-row groups 1024 B apart
// (SBO), LBO unused. MN-major: 64-element MN atoms `lbo` bytes apart, 8-row
// K groups `sbo` bytes apart. Tile bases must be 1024-byte aligned.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr) { return sw128_desc(saddr, 16, 1024); }

// Instruction descriptor, kind::f16: fp32 accumulator, A/B fp16 (fmt 0) or
// bf16 (fmt 1), M x N tile, A/B major-ness (0 = K-major, 1 = MN-major).
__host__ __device__ constexpr uint32_t idesc_f16(int ab_fmt, int m, int n, int a_mn_major,
                                                 int b_mn_major) {
  return (1u << 4)                                   // D format: f32
         | (static_cast<uint32_t>(ab_fmt) << 7)      // A format
         | (static_cast<uint32_t>(ab_fmt) << 10)     // B format
         | (static_cast<uint32_t>(a_mn_major) << 15) // A major
         | (static_cast<uint32_t>(b_mn_major) << 16) // B major
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

// byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a
// 128B-swizzled tile whose rows are 128 bytes
__device__ __forceinline__ uint32_t sw128_off(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// same for a 64-byte-swizzled tile with 64-byte rows (chunk 0..3)
__device__ __forceinline__ uint32_t sw64_off(uint32_t row, uint32_t chunk) {
  return row * 64u + ((chunk ^ ((row >> 1) & 3u)) << 4);
}

// 8 x 16-bit values (fp16, or bf16 when `bf16`) -> fp32
__device__ __forceinline__ void unpack8(const uint4& r, int bf16, float (&f)[8]) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float2 v;
    if (bf16) {
      __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[e]);
      v = __bfloat1622float2(h);
    } else {
      __half2 h = *reinterpret_cast<const __half2*>(&w[e]);
      v = __half22float2(h);
    }
    f[2 * e] = v.x;
    f[2 * e + 1] = v.y;
  }
}

// -------------------------------------------------------------- small math
// logistic function with the fast exp2-based exponential and approximate divide
// (relative error ~1e-7, far below the fp16 storage rounding that follows)
__device__ __forceinline__ float sigmoidf_fast(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

// Logistic function using ONE special-function (MUFU) op: e = 2^(-x log2 e) on the
// MUFU pipe, then 1/(1+e) by Newton-Raphson on the FMA pipe. Seed: the classic
// exponent-reflection estimate r0 = bits(0x7EF311C3 - bits(d)) (relative error
// < 1/8 for normal d), refined by three steps r <- r + r(1 - d r) (quadratic
// convergence: 1/8 -> 1.6e-2 -> 2.4e-4 -> ~6e-8). x is clamped to [-60, 60], where
// the logistic is 0 or 1 to far below fp16 resolution, so d stays a normal float.
// The epilogues are MUFU-throughput-bound (16 ops/clk/SM), so this halves their cost.
__device__ __forceinline__ float sigmoid_nr(float x) {
  x = fminf(fmaxf(x, -60.0f), 60.0f);
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * -1.4426950408889634f));
  const float d = 1.0f + e;
  float r = __int_as_float(0x7EF311C3 - __float_as_int(d));
#pragma unroll
  for (int i = 0; i < 3; ++i) r = fmaf(r, fmaf(-d, r, 1.0f), r);
  return r;
}

// tanh on the special-function unit (PTX tanh.approx.f32, one MUFU op)
__device__ __forceinline__ float tanh_mufu(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// p * sigmoid(g) with sigmoid(g) = 0.5 + 0.5 tanh(g / 2): one MUFU op and three
// FP32 ops per element (the epilogues are bound by FP32 issue and MUFU throughput)
__device__ __forceinline__ float gated_tanh(float p, float g) {
  const float hp = 0.5f * p;
  return fmaf(hp, tanh_mufu(0.5f * g), hp);
}

// same with both arguments already halved: hp = p / 2, hg = g / 2
__device__ __forceinline__ float gated_tanh_half(float hp, float hg) {
  return fmaf(hp, tanh_mufu(hg), hp);
}

// two lanes of the same at once: FFMA2 (sm_100 packed fp32, IEEE round-to-nearest per
// lane) for the affine part, two MUFU tanh
__device__ __forceinline__ float2 gated_tanh_half2(float2 hp, float2 hg) {
  return __ffma2_rn(hp, make_float2(tanh_mufu(hg.x), tanh_mufu(hg.y)), hp);
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_bf162(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Position tiling shared by the input and output stages: 128 positions per
// tile arranged as U_T rows x V_T columns of the (R x S) position grid.
struct PosTiling {
  int R, S, B;      // grid rows, columns, batches
  int vt, ut;       // tile shape (vt * ut == 128), vt in {64, 128}
  int tiles_u, tiles_v, tiles;
  int pf;           // L2 prefetch distance of the stage producers, in own tiles (0: off)
  __host__ __device__ void init(int batch, int rows, int cols) {
    pf = 0;
    B = batch;
    R = rows;
    S = cols;
    vt = cols > 64 ? 128 : 64;
    ut = 128 / vt;
    tiles_u = (rows + ut - 1) / ut;
    tiles_v = (cols + vt - 1) / vt;
    tiles = batch * tiles_u * tiles_v;
  }
  // tile id -> (b, u0, v0)
  __host__ __device__ void tile(int t, int& b, int& u0, int& v0) const {
    const int per_b = tiles_u * tiles_v;
    b = t / per_b;
    const int r = t - b * per_b;
    u0 = (r / tiles_v) * ut;
    v0 = (r % tiles_v) * vt;
  }
};

}  // namespace ftm
