// Shared helpers for the sm_100a SunShape kernels: status plumbing, dispatch
// counters, fp16 conversions and thin inline-PTX wrappers (mbarrier, bulk and
// tensor TMA copies, ldmatrix, warp MMA).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/sunshape_b200.h"

namespace ss {

// ---------------------------------------------------------------- host side
int fail(int code, const std::string& msg);      // records msg, returns code
int check_launch(const char* what);              // cudaGetLastError -> status
void count_dispatch(const char* name);
int sm_count();                                  // of the current device
// Device address of the process error sink (ss_set_error_sink), or null.
int* error_sink();

#define SS_REQUIRE(cond, msg)                                  \
  do {                                                         \
    if (!(cond)) return ::ss::fail(SS_ERR_BAD_ARG, (msg));     \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Creates (or returns a cached) 3-D tiled tensor map over fp16 data laid out
// as pairs x rows x inner (inner contiguous, rows packed, pairs strided by
// pair_stride_bytes) with a box of box_inner x box_rows x 1 and 128-byte
// swizzle. Returns nullptr on failure (message recorded).
const CUtensorMap* tmap_3d_f16_sw128(const void* base, uint64_t inner, uint64_t rows,
                                     uint64_t pairs, uint64_t pair_stride_bytes,
                                     uint32_t box_inner, uint32_t box_rows);
// Same for any key dtype (SS_F16 / SS_BF16 / SS_F32) and an explicit row
// stride (bytes): dims inner x rows x pairs.
const CUtensorMap* tmap_3d_sw128(const void* base, int dtype, uint64_t inner, uint64_t rows,
                                 uint64_t pairs, uint64_t row_stride_bytes,
                                 uint64_t pair_stride_bytes, uint32_t box_inner,
                                 uint32_t box_rows);

// ---------------------------------------------------------------- device side
__device__ __forceinline__ float h2f(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ uint16_t f2h(float f) {
  return __half_as_ushort(__float2half_rn(f));
}
__device__ __forceinline__ float bf2f(uint16_t h) {
  return __bfloat162float(__ushort_as_bfloat16(h));
}

// Loads element i of a row of dtype dt as float.
__device__ __forceinline__ float load_as_f32(const void* p, int dt, int64_t i) {
  if (dt == SS_F32) return reinterpret_cast<const float*>(p)[i];
  const uint16_t u = reinterpret_cast<const uint16_t*>(p)[i];
  return dt == SS_F16 ? h2f(u) : bf2f(u);
}

// Rounds a float to the value representable in dtype dt (float result).
__device__ __forceinline__ float round_to(float x, int dt) {
  if (dt == SS_F16) return __half2float(__float2half_rn(x));
  if (dt == SS_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  return x;
}

__device__ __forceinline__ void store_from_f32(void* p, int dt, int64_t i, float v) {
  if (dt == SS_F32) {
    reinterpret_cast<float*>(p)[i] = v;
  } else if (dt == SS_F16) {
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  } else {
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  }
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// One potentially-blocking probe of a barrier phase: the warp may be
// suspended for up to ~0.5 ms waiting for the phase instead of spinning.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(500000u)
      : "memory");
  return ok != 0;
}
// Non-blocking probe of a barrier phase.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: polls the barrier phase and gives up (returns false) once
// `limit_ns` nanoseconds of %globaltimer have passed.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > limit_ns) return false;
  }
}

// A bounded wait gave up: OR `code` into the launch's error word and, when a
// process error sink is attached, into that host word (system scope, so the
// host sees it without synchronizing).
__device__ __forceinline__ void report_wait_failure(int* ws_err, int* sink, int code) {
  if (ws_err) atomicOr(ws_err, code);
  if (sink) atomicOr_system(sink, code);
}

// ---- bulk / tensor TMA (no cluster multicast anywhere in this library) ------
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst_smem, const CUtensorMap* map, int32_t x,
                                            int32_t y, int32_t z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst_smem)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
// 16-byte global -> shared copy (generic proxy, L2 only); src_bytes < 16
// zero-fills the rest (0 = all zeros, nothing read).
__device__ __forceinline__ void cp_async16(uint32_t dst_smem, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst_smem), "l"(src),
               "r"(src_bytes)
               : "memory");
}
// Arrives on the barrier once all of this thread's earlier cp.async copies
// have landed (the arrival counts toward the barrier's expected count).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// Programmatic dependent launch: the primary grid allows its dependent to be
// scheduled; the dependent waits for the primary's completion and memory.
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// subsequent async-proxy (bulk copy) writes to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- named barriers ---------------------------------------------------------
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- ldmatrix / mma ---------------------------------------------------------
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_trans(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}
// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col)
__device__ __forceinline__ void mma_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// (a, b) += (x, y) as one packed fp32 add (two round-to-nearest fp32 adds).
__device__ __forceinline__ void add_f32x2(float& a, float& b, float x, float y) {
  asm("{\n .reg .b64 t, u;\n mov.b64 t, {%0, %1};\n mov.b64 u, {%2, %3};\n"
      " add.rn.f32x2 t, t, u;\n mov.b64 {%0, %1}, t;\n}"
      : "+f"(a), "+f"(b)
      : "f"(x), "f"(y));
}

// (a, b) *= s as one packed fp32 multiply (round to nearest).
__device__ __forceinline__ void mul_f32x2(float& a, float& b, float s) {
  asm("{\n .reg .b64 t, u;\n mov.b64 t, {%0, %1};\n mov.b64 u, {%2, %2};\n"
      " mul.rn.f32x2 t, t, u;\n mov.b64 {%0, %1}, t;\n}"
      : "+f"(a), "+f"(b)
      : "f"(s));
}

// (a, b) = (a, b) * s + z with packed fp32 ops, a multiply then an add, as
// the reference computes q * scale + zero in fp32 (two roundings).
__device__ __forceinline__ void mul_add_f32x2(float& a, float& b, float s, float z) {
  asm("{\n .reg .b64 t, u;\n mov.b64 t, {%0, %1};\n mov.b64 u, {%2, %2};\n"
      " mul.rn.f32x2 t, t, u;\n mov.b64 u, {%3, %3};\n add.rn.f32x2 t, t, u;\n"
      " mov.b64 {%0, %1}, t;\n}"
      : "+f"(a), "+f"(b)
      : "f"(s), "f"(z));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace ss
