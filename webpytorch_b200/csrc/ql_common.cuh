// Shared device helpers for the quantized-linear kernels (sm_100a only).
//
// Everything here is written from the PTX ISA: integer-to-fp16 "magic number" unpacking,
// the legacy warp-level mma.sync used by the decode GEMV (its operands live in registers,
// which is what a bandwidth-bound GEMV wants), and small load/convert helpers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/qlinear.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "webpytorch_b200 kernels are written for sm_100a only"
#endif

namespace ql {

// ---------------------------------------------------------------------------------------
// error reporting shared by every translation unit of the library
// ---------------------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int cuda_status(cudaError_t e, const char* where);

// Launch flags set through ql_set_launch_flags (QL_LAUNCH_* bits).
int launch_flags();

// Stream-ordered scratch allocation (cudaMallocAsync) for calls given too small a workspace;
// fails with QL_ERR_UNSUPPORTED while an AllocGuard is alive on the calling thread.
int stream_alloc(void** p, size_t bytes, cudaStream_t st, const char* what);
struct AllocGuard {
  AllocGuard();
  ~AllocGuard();
  bool prev;
};

// Integer knob from the environment (benchmark tuning only), read once per name by the caller.
int env_int(const char* name, int dflt);

// ---------------------------------------------------------------------------------------
// bit twiddling
// ---------------------------------------------------------------------------------------
// (a & b) | c in one LOP3 (truth table 0xEA for a=0xF0, b=0xCC, c=0xAA).
__device__ __forceinline__ uint32_t lop3_andor(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }

// fp16 0x6400 is 1024.0; OR-ing a value v < 1024 into its low mantissa bits gives 1024 + v
// exactly, because fp16 has unit spacing on [1024, 2048).
constexpr uint32_t kMagicF16x2 = 0x64006400u;

// ---------------------------------------------------------------------------------------
// legacy warp MMA: D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col)
// ---------------------------------------------------------------------------------------
// Not volatile: a pure register computation the compiler may schedule freely, so independent
// loads and unpacking interleave with the MMAs.
__device__ __forceinline__ void mma_16816_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------------------
// global loads that bypass L1 allocation for streamed, read-once weights
// ---------------------------------------------------------------------------------------
// Weights are read-only for the kernel's lifetime, so these loads are not volatile: the
// compiler may hoist them and overlap them with unrelated work.
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ldg_stream_v2(const void* p) {
  uint2 r;
  asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

// ---------------------------------------------------------------------------------------
// programmatic dependent launch (PDL) and cluster barriers
// ---------------------------------------------------------------------------------------
// Lets the next kernel in the stream be scheduled once every CTA of this grid has run it.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Waits until the previous kernel in the stream has completed and its writes are visible
// (a no-op when this grid was not launched as a programmatic dependent).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------------------
// dtype helpers
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ float load_as_float(const void* base, int dtype, long idx) {
  switch (dtype) {
    case QL_F16: return __half2float(reinterpret_cast<const __half*>(base)[idx]);
    case QL_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
    default: return reinterpret_cast<const float*>(base)[idx];
  }
}

__device__ __forceinline__ void store_from_float(void* base, int dtype, long idx, float v) {
  switch (dtype) {
    case QL_F16: reinterpret_cast<__half*>(base)[idx] = __float2half_rn(v); break;
    case QL_BF16: reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v); break;
    default: reinterpret_cast<float*>(base)[idx] = v; break;
  }
}

// Exact power-of-two scale 2^e (|e| small) without touching the math library.
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((e + 127) << 23); }

// Exponent e such that m * 2^-e lies in [2^14, 2^15): staging a row of activations as fp16
// with this scale keeps every value in range and loses nothing but the (exact) exponent shift.
__device__ __forceinline__ int stage_exponent(float absmax) {
  if (!(absmax > 0.f) || !(absmax < 3.0e38f)) return 0;   // zero / inf / nan rows: no scaling
  int be = ((__float_as_int(absmax) >> 23) & 0xff) - 127;  // floor(log2(absmax)) for normals
  if (be < -126) be = -126;
  int e = be - 14;
  if (e < -100) e = -100;
  if (e > 100) e = 100;
  return e;
}

// Exponent e such that m * 2^-e lies in [2^13, 2^14): activations staged as integers
// rint(x * 2^-e) then fit 15 bits (|v| <= 2^14), which two signed bytes hold as 256 * hi + lo.
// Clamped so that both 2^e and 2^-e are normal floats; zero / non-finite rows get 0.
__device__ __forceinline__ int stage_exponent_i15(float absmax) {
  if (!(absmax > 0.f) || !(absmax < 3.0e38f)) return 0;
  int be = ((__float_as_int(absmax) >> 23) & 0xff) - 127;  // floor(log2(absmax)) for normals
  int e = be - 13;
  if (e < -110) e = -110;
  if (e > 114) e = 114;
  return e;
}

// integer MMA: D(16x8 s32) += A(16x32 u8, row) * B(32x8 s8, col)
__device__ __forceinline__ void mma_16832_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 6-bit scale and min of sub-block j from the 12 scale bytes held in three words
// s0 = bytes 0..3, s1 = bytes 4..7, s2 = bytes 8..11 (get_scale_min_k4).
__device__ __forceinline__ void q4k_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j, uint32_t& sc,
                                              uint32_t& m) {
  if (j < 4) {
    sc = (s0 >> (8 * j)) & 63u;
    m = (s1 >> (8 * j)) & 63u;
  } else {
    const int i = j - 4;
    sc = ((s2 >> (8 * i)) & 0x0Fu) | (((s0 >> (8 * i + 6)) & 3u) << 4);
    m = ((s2 >> (8 * i + 4)) & 0x0Fu) | (((s1 >> (8 * i + 6)) & 3u) << 4);
  }
}

}  // namespace ql
