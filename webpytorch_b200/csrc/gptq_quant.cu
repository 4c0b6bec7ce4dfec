// GPTQ-format quantiser on the GPU: asymmetric min/max group quantisation of a dense weight and
// packing into the AutoGPTQ layout (or the reference's own packing), for quantize-on-load and
// for writing AutoGPTQ checkpoints.
//
// Reference semantics (webtorch/quantize.py:80-106, _quantize_raw and _pack_autogptq; the same
// arithmetic as _gptq_quantize, webtorch/_core.py:3782-3824, in float32):
//   W (out, in) is used transposed as (in, out) = (K, N), zero-padded to Kp = K + (-K % gs) and
//   Np = N + (-N % per); per group g of gs rows and column n:
//     lo, hi = min, max;  s = (hi - lo) / qmax (1e-8 when 0);  z = clip(rint(-lo / s), 0, qmax)
//     q[k, n] = clip(rint(W[k, n] / s) + z, 0, qmax)
//   qweight [Kp/per, Np] packs per values LSB-first along K, qzeros [Kp/gs, Np/per] packs
//   (z - zero_store_offset) & qmax LSB-first along N (offset 1: AutoGPTQ stores zp - 1),
//   scales [Kp/gs, Np] as fp32 or rounded to fp16.
// Every step is an IEEE float32 operation with round-to-nearest-even, as numpy's, so the packed
// output is bit-identical to the reference's.
#include "ql_common.cuh"

namespace ql {
namespace {

constexpr int kCols = 32;     // columns per CTA
constexpr int kThreads = 256;

// One CTA per (group, 32 columns): the group's [gs][32] tile goes through shared memory.
__global__ void __launch_bounds__(kThreads) gptq_quantize_kernel(const void* __restrict__ W, int w_dtype, long ldw,
                                                                 int N, int K, int gs, int bits, int zstore,
                                                                 uint32_t* __restrict__ qweight,
                                                                 uint32_t* __restrict__ qzeros,
                                                                 void* __restrict__ scales, int sc_dtype, int Np) {
  extern __shared__ float tile[];   // [gs][kCols + 1]
  __shared__ float s_scale[kCols];
  __shared__ int s_zero[kCols];
  const int g = blockIdx.y, n0 = blockIdx.x * kCols;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = 32 / bits, qmax = (1 << bits) - 1;
  const int k0 = g * gs;
  // load: warp w reads rows n0 + w, n0 + w + 8, ... of W (contiguous along K), transposed
  for (int c = warp; c < kCols; c += kThreads / 32) {
    const int n = n0 + c;
    for (int kk = lane; kk < gs; kk += 32) {
      const int k = k0 + kk;
      float v = 0.f;
      if (n < N && k < K) v = load_as_float(W, w_dtype, (long)n * ldw + k);
      tile[kk * (kCols + 1) + c] = v;
    }
  }
  __syncthreads();
  // per column: min / max over the group, scale and zero point (8 threads per column)
  {
    const int c = tid >> 3, part = tid & 7;
    float lo = 3.4e38f, hi = -3.4e38f;
    for (int kk = part; kk < gs; kk += 8) {
      const float v = tile[kk * (kCols + 1) + c];
      lo = fminf(lo, v);
      hi = fmaxf(hi, v);
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if (part == 0) {
      float s = __fdiv_rn(__fsub_rn(hi, lo), (float)qmax);
      if (s == 0.f) s = 1e-8f;
      float z = rintf(__fdiv_rn(-lo, s));
      z = fminf(fmaxf(z, 0.f), (float)qmax);
      s_scale[c] = s;
      s_zero[c] = (int)z;
    }
  }
  __syncthreads();
  // quantise in place (the tile then holds q as floats)
  for (int i = tid; i < gs * kCols; i += kThreads) {
    const int kk = i / kCols, c = i - kk * kCols;
    float* p = &tile[kk * (kCols + 1) + c];
    const float q = rintf(__fdiv_rn(*p, s_scale[c])) + (float)s_zero[c];
    *p = fminf(fmaxf(q, 0.f), (float)qmax);
  }
  __syncthreads();
  // qweight: packed row r of the group = values k0 + r * per .. + per - 1 of each column
  const int rows = gs / per;
  for (int i = tid; i < rows * kCols; i += kThreads) {
    const int r = i / kCols, c = i - r * kCols;
    const int n = n0 + c;
    if (n >= Np) continue;
    uint32_t w = 0u;
    for (int j = 0; j < per; ++j) w |= ((uint32_t)tile[(r * per + j) * (kCols + 1) + c] & (uint32_t)qmax) << (bits * j);
    qweight[(long)(k0 / per + r) * Np + n] = w;
  }
  // qzeros: per columns per word, LSB-first along N; scales
  if (tid < kCols / per) {
    const int nw0 = n0 + tid * per;
    if (nw0 < Np) {
      uint32_t w = 0u;
      for (int j = 0; j < per; ++j) w |= ((uint32_t)(s_zero[tid * per + j] - zstore) & (uint32_t)qmax) << (bits * j);
      qzeros[(long)g * (Np / per) + nw0 / per] = w;
    }
  }
  if (tid < kCols && n0 + tid < Np) {
    const long o = (long)g * Np + n0 + tid;
    if (sc_dtype == QL_F16)
      reinterpret_cast<__half*>(scales)[o] = __float2half_rn(s_scale[tid]);
    else
      reinterpret_cast<float*>(scales)[o] = s_scale[tid];
  }
}

}  // namespace
}  // namespace ql

using namespace ql;

extern "C" int ql_gptq_quantize(const void* W, int w_dtype, long ldw, int N, int K, int gs, int bits,
                                int zero_store_offset, int32_t* qweight, int32_t* qzeros, void* scales,
                                int scales_dtype, void* stream) {
  if (bits != 4 && bits != 8) {
    set_error("ql_gptq_quantize: bits must be 4 or 8 (got %d)", bits);
    return QL_ERR_UNSUPPORTED;
  }
  const int per = 32 / bits;
  if (!W || !qweight || !qzeros || !scales || N <= 0 || K <= 0 || gs <= 0 || gs % per != 0 || gs > 1024 ||
      ldw < K || (zero_store_offset != 0 && zero_store_offset != 1) ||
      (w_dtype != QL_F32 && w_dtype != QL_F16 && w_dtype != QL_BF16) ||
      (scales_dtype != QL_F32 && scales_dtype != QL_F16)) {
    set_error("ql_gptq_quantize: bad arguments (N=%d K=%d gs=%d bits=%d ldw=%ld; gs a multiple of %d, <= 1024)", N,
              K, gs, bits, ldw, per);
    return QL_ERR_ARG;
  }
  const int Kp = K + (gs - K % gs) % gs;
  const int Np = N + (per - N % per) % per;
  const dim3 grid((Np + kCols - 1) / kCols, Kp / gs);
  const size_t smem = (size_t)gs * (kCols + 1) * sizeof(float);
  cudaStream_t st = (cudaStream_t)stream;
  if (smem > 48 * 1024) {
    const int rc = cuda_status(cudaFuncSetAttribute(gptq_quantize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    (int)smem),
                               "ql_gptq_quantize: cudaFuncSetAttribute");
    if (rc) return rc;
  }
  gptq_quantize_kernel<<<grid, kThreads, smem, st>>>(W, w_dtype, ldw, N, K, gs, bits, zero_store_offset,
                                                     reinterpret_cast<uint32_t*>(qweight),
                                                     reinterpret_cast<uint32_t*>(qzeros), scales, scales_dtype, Np);
  return cuda_status(cudaGetLastError(), "ql_gptq_quantize launch");
}
