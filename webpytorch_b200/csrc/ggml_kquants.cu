// GGUF Q8_0, Q5_K and Q6_K weights on the GPU: exact dequantisation, and a decode GEMV that
// reads the file's blocks in place (no load-time re-layout) and decodes them inside the matmul.
//
// Block formats (webtorch/ggufload.py:140-145, 210-246; values of an [N, K] weight stored as N
// rows of K/block blocks):
//   Q8_0  32 values / 34 bytes: f16 d | int8 qs[32];                       w = d * q
//   Q5_K  256 values / 176 bytes: f16 d | f16 dmin | scales[12] (6-bit scale / min per 32-value
//         sub-block, packed as Q4_K's) | qh[32] (5th bits) | qs[128] (low nibbles):
//         sub-block j = 2g + u takes the low (u = 0) or high (u = 1) nibbles of qs[32g .. 32g+31]
//         plus 16 * bit j of qh[i];                                         w = d*sc_j*q - dmin*m_j
//   Q6_K  256 values / 210 bytes: ql[128] | qh[64] | int8 scales[16] | f16 d: value 128h + 32t + l
//         (h < 2, t < 4, l < 32) is (ql[64h + l + 32(t & 1)] >> 4(t >> 1) & 15) | ((qh[32h + l] >>
//         2t) & 3) << 4, minus 32, times d * scales[8h + l/16 + 2t]
// The dequantisers round exactly as numpy does the reference's expressions: (d*sc)*q for Q6_K,
// d*q for Q8_0, (d*sc*q) - (dmin*m) for Q5_K (every product but the last step is exact in fp32).
//
// GEMV: one warp per weight row, a CTA of 8 warps covers 8 rows and up to 4 tokens. The K range
// is walked in chunks whose activations are staged once per CTA as fp32 in shared memory; each
// warp copies its row's blocks for the chunk into its own shared-memory slots with 4-byte
// cp.async copies (double-buffered), then every lane decodes 8 consecutive values per 256 and
// accumulates x * q per scale run in fp32, folding scale and min once per run.
#include "ql_common.cuh"

namespace ql {
namespace {

enum { kQ8_0 = 8, kQ4_K = 12, kQ5_K = 13, kQ6_K = 14 };

// copy unit: UV values in UB bytes (4-byte aligned whenever a row is), stored in smem slots of SB
template <int T>
struct Fmt;
template <>
struct Fmt<kQ8_0> {
  static constexpr int UV = 256, UB = 272, SB = 272, BB = 34;
};
template <>
struct Fmt<kQ5_K> {
  static constexpr int UV = 256, UB = 176, SB = 176, BB = 176;
};
template <>
struct Fmt<kQ6_K> {
  static constexpr int UV = 512, UB = 420, SB = 432, BB = 210;
};

__device__ __forceinline__ float f16_at(const unsigned char* p) {
  return __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(p)));
}
// 8 bytes at a 2-byte aligned shared-memory address
__device__ __forceinline__ uint2 ld8_u16(const unsigned char* p) {
  const unsigned short* s = reinterpret_cast<const unsigned short*>(p);
  return make_uint2((uint32_t)s[0] | ((uint32_t)s[1] << 16), (uint32_t)s[2] | ((uint32_t)s[3] << 16));
}

// Q4_K / Q5_K 6-bit scale and min of sub-block j from the 12 packed bytes (get_scale_min_k4)
__device__ __forceinline__ void scale_min_k4(const unsigned char* s, int j, int& sc, int& m) {
  if (j < 4) {
    sc = s[j] & 63;
    m = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
    m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// ------------------------------------------------------------------ exact dequantisation
// One thread per 8 consecutive values of a 256-value run (Q8_0: of 8 blocks).
template <int T>
__global__ void __launch_bounds__(256) ggml_dequant_kernel(const uint8_t* __restrict__ raw, float* __restrict__ W,
                                                           long nruns) {
  using F = Fmt<T>;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nruns * 32; i += (long)gridDim.x * blockDim.x) {
    const long run = i >> 5;
    const int l = (int)(i & 31);
    float* o = W + run * 256 + 8 * l;
    if constexpr (T == kQ8_0) {
      const uint8_t* b = raw + (run * 8 + (l >> 2)) * F::BB;
      const float d = __half2float(__ushort_as_half((unsigned short)(b[0] | (b[1] << 8))));
      const int8_t* q = reinterpret_cast<const int8_t*>(b + 2 + 8 * (l & 3));
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = __fmul_rn(d, (float)q[j]);
    } else if constexpr (T == kQ5_K) {
      const uint8_t* b = raw + run * F::BB;
      const float d = __half2float(__ushort_as_half((unsigned short)(b[0] | (b[1] << 8))));
      const float dmin = __half2float(__ushort_as_half((unsigned short)(b[2] | (b[3] << 8))));
      const int g = l >> 3, u = (l >> 2) & 1, p = 8 * (l & 3), j = 2 * g + u;
      int sc, m;
      scale_min_k4(b + 4, j, sc, m);
      const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int qs = b[48 + 32 * g + p + k];
        const int q = (u ? (qs >> 4) : (qs & 15)) + (((b[16 + p + k] >> j) & 1) << 4);
        o[k] = __fsub_rn(__fmul_rn(d1, (float)q), m1);
      }
    } else {
      const uint8_t* b = raw + run * F::BB;
      const float d = __half2float(__ushort_as_half((unsigned short)(b[208] | (b[209] << 8))));
      const int h = l >> 4, t = (l >> 2) & 3, lo = 8 * (l & 3);
      const float ds = __fmul_rn(d, (float)(int8_t)b[192 + 8 * h + (lo >> 4) + 2 * t]);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int ql = b[64 * h + 32 * (t & 1) + lo + k];
        const int q = (((t >> 1) ? (ql >> 4) : (ql & 15)) | (((b[128 + 32 * h + lo + k] >> (2 * t)) & 3) << 4)) - 32;
        o[k] = __fmul_rn(ds, (float)q);
      }
    }
  }
}

// ------------------------------------------------------------------ decode GEMV
constexpr int kWarps = 8;
constexpr int kChunk = 2048;   // K values per activation chunk
constexpr int kMaxT = 4;       // tokens per CTA

struct GemvArgs {
  const void* x;
  int x_dtype;
  long ldx;
  const uint8_t* raw;
  long row_bytes;
  const float* bias;
  void* out;
  int out_dtype;
  long ldo;
  int M, K, N;
};

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Lane l's share of one 256-value run held in shared memory at b: 8 values, their token dot
// products accumulated into acc[MT] with the run's scales folded in.
template <int T, int MT>
__device__ __forceinline__ void run_dot(const unsigned char* b, int l, const float* xs, int xstride, float (&acc)[MT]) {
  const float* xv = xs + 8 * l;   // x of this lane's 8 values (token 0; tokens xstride apart)
  float w[8];
  float scale, bias_m = 0.f;      // sum x*w = scale * sum x*q - bias_m * sum x
  if constexpr (T == kQ8_0) {
    const unsigned char* blk = b + (l >> 2) * 34;
    scale = f16_at(blk);
    const uint2 q = ld8_u16(blk + 2 + 8 * (l & 3));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      w[k] = (float)(int8_t)(q.x >> (8 * k));
      w[4 + k] = (float)(int8_t)(q.y >> (8 * k));
    }
  } else if constexpr (T == kQ5_K) {
    const int g = l >> 3, u = (l >> 2) & 1, p = 8 * (l & 3), j = 2 * g + u;
    int sc, m;
    scale_min_k4(b + 4, j, sc, m);
    scale = f16_at(b) * (float)sc;
    bias_m = f16_at(b + 2) * (float)m;
    const uint2 qs = *reinterpret_cast<const uint2*>(b + 48 + 32 * g + p);
    const uint2 qh = *reinterpret_cast<const uint2*>(b + 16 + p);
    const uint32_t lo0 = u ? (qs.x >> 4) & 0x0F0F0F0Fu : qs.x & 0x0F0F0F0Fu;
    const uint32_t lo1 = u ? (qs.y >> 4) & 0x0F0F0F0Fu : qs.y & 0x0F0F0F0Fu;
    const uint32_t h0 = ((qh.x >> j) & 0x01010101u) << 4, h1 = ((qh.y >> j) & 0x01010101u) << 4;
    const uint32_t q0 = lo0 | h0, q1 = lo1 | h1;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      w[k] = (float)((q0 >> (8 * k)) & 0xFF);
      w[4 + k] = (float)((q1 >> (8 * k)) & 0xFF);
    }
  } else {
    const int h = l >> 4, t = (l >> 2) & 3, lo = 8 * (l & 3);
    scale = f16_at(b + 208) * (float)(int8_t)b[192 + 8 * h + (lo >> 4) + 2 * t];
    const uint2 ql = ld8_u16(b + 64 * h + 32 * (t & 1) + lo);
    const uint2 qh = ld8_u16(b + 128 + 32 * h + lo);
    const int sh = 4 * (t >> 1);
    const uint32_t q0 = ((ql.x >> sh) & 0x0F0F0F0Fu) | (((qh.x >> (2 * t)) & 0x03030303u) << 4);
    const uint32_t q1 = ((ql.y >> sh) & 0x0F0F0F0Fu) | (((qh.y >> (2 * t)) & 0x03030303u) << 4);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      w[k] = (float)((int)((q0 >> (8 * k)) & 0xFF) - 32);
      w[4 + k] = (float)((int)((q1 >> (8 * k)) & 0xFF) - 32);
    }
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const float4 xa = *reinterpret_cast<const float4*>(xv + m * xstride);
    const float4 xb = *reinterpret_cast<const float4*>(xv + m * xstride + 4);
    float s = xa.x * w[0];
    s = fmaf(xa.y, w[1], s);
    s = fmaf(xa.z, w[2], s);
    s = fmaf(xa.w, w[3], s);
    s = fmaf(xb.x, w[4], s);
    s = fmaf(xb.y, w[5], s);
    s = fmaf(xb.z, w[6], s);
    s = fmaf(xb.w, w[7], s);
    acc[m] = fmaf(scale, s, acc[m]);
    if constexpr (T == kQ5_K) {
      const float sx = ((xa.x + xa.y) + (xa.z + xa.w)) + ((xb.x + xb.y) + (xb.z + xb.w));
      acc[m] = fmaf(-bias_m, sx, acc[m]);
    }
  }
}

template <int T, int MT>
__global__ void __launch_bounds__(kWarps * 32) ggml_gemv_kernel(const GemvArgs a) {
  using F = Fmt<T>;
  constexpr int UPC = kChunk / F::UV;     // copy units per chunk and row
  extern __shared__ __align__(16) unsigned char smem[];
  float* xs = reinterpret_cast<float*>(smem);                                 // [MT][kChunk]
  unsigned char* slots = smem + (size_t)MT * kChunk * 4;                      // [warps][2][UPC][SB]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = blockIdx.x * kWarps + warp;
  const int m0 = blockIdx.y * kMaxT;
  const int M = min(MT, a.M - m0);
  const bool row_ok = n < a.N;
  unsigned char* my = slots + (size_t)warp * 2 * UPC * F::SB;
  const uint8_t* rowp = a.raw + (size_t)(row_ok ? n : 0) * a.row_bytes;
  const int nchunk = (a.K + kChunk - 1) / kChunk;
  // copy the row's units of chunk c into buffer c & 1 (4-byte cp.async, coalesced over lanes)
  auto issue = [&](int c) {
    const int k0 = c * kChunk;
    const int units = min(UPC, (a.K - k0) / F::UV);
    unsigned char* dst = my + (c & 1) * UPC * F::SB;
    const uint8_t* src = rowp + (size_t)(k0 / F::UV) * F::UB;
    if (row_ok) {
      for (int uu = 0; uu < units; ++uu)
        for (int wd = lane; wd < F::UB / 4; wd += 32)
          cp_async4(static_cast<uint32_t>(__cvta_generic_to_shared(dst + uu * F::SB + 4 * wd)), src + uu * F::UB + 4 * wd);
    }
    cp_async_commit();
  };
  float acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0.f;
  issue(0);
  for (int c = 0; c < nchunk; ++c) {
    const int k0 = c * kChunk;
    const int klen = min(kChunk, a.K - k0);
    __syncthreads();   // the previous chunk's activations are no longer read
    for (int i = tid; i < MT * klen; i += kWarps * 32) {
      const int m = i / klen, k = i - m * klen;
      xs[m * kChunk + k] = m < M ? load_as_float(a.x, a.x_dtype, (long)(m0 + m) * a.ldx + k0 + k) : 0.f;
    }
    if (c + 1 < nchunk) issue(c + 1);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();   // activations staged, this warp's units landed
    const unsigned char* buf = my + (c & 1) * UPC * F::SB;
    const int units = klen / F::UV;
    for (int uu = 0; uu < units; ++uu) {
      const unsigned char* u = buf + uu * F::SB;
#pragma unroll
      for (int r = 0; r < F::UV / 256; ++r)
        run_dot<T, MT>(u + r * (F::UV == 512 ? 210 : 0), lane, xs + uu * F::UV + r * 256, kChunk, acc);
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    float v = acc[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0 && row_ok && m < M) {
      if (a.bias) v += a.bias[n];
      store_from_float(a.out, a.out_dtype, (long)(m0 + m) * a.ldo + n, v);
    }
  }
}

template <int T>
int launch_gemv(const GemvArgs& a, cudaStream_t st) {
  using F = Fmt<T>;
  constexpr int UPC = kChunk / F::UV;
  const dim3 grid((a.N + kWarps - 1) / kWarps, (a.M + kMaxT - 1) / kMaxT);
  const size_t slots = (size_t)kWarps * 2 * UPC * F::SB;
  static int configured_dev[3] = {-1, -1, -1};
  int dev = 0;
  cudaGetDevice(&dev);
  auto go = [&](auto kern, int mt, int slot) {
    const size_t smem = (size_t)mt * kChunk * 4 + slots;
    if (configured_dev[slot] != dev) {
      const int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                                 "ql_ggml_matmul: cudaFuncSetAttribute");
      if (rc) return rc;
      configured_dev[slot] = dev;
    }
    kern<<<grid, kWarps * 32, smem, st>>>(a);
    return cuda_status(cudaGetLastError(), "ggml_gemv launch");
  };
  if (a.M == 1) return go(ggml_gemv_kernel<T, 1>, 1, 0);
  if (a.M == 2) return go(ggml_gemv_kernel<T, 2>, 2, 1);
  return go(ggml_gemv_kernel<T, kMaxT>, kMaxT, 2);
}

bool type_info(int t, int& vals, int& bytes) {
  switch (t) {
    case kQ8_0: vals = 32; bytes = 34; return true;
    case kQ4_K: vals = 256; bytes = 144; return true;
    case kQ5_K: vals = 256; bytes = 176; return true;
    case kQ6_K: vals = 256; bytes = 210; return true;
    default: return false;
  }
}

}  // namespace
}  // namespace ql

using namespace ql;

extern "C" int ql_q4k_dequant(const uint8_t* raw, float* W, int N, int K, void* stream);
extern "C" int ql_q4k_matmul(const void* x, int x_dtype, long ldx, const uint8_t* raw, const float* bias, void* out,
                             int out_dtype, long ldo, int M, int K, int N, void* stream);

extern "C" int ql_ggml_dequant(int ggml_type, const uint8_t* raw, float* W, int N, int K, void* stream) {
  int vals, bytes;
  if (!type_info(ggml_type, vals, bytes)) {
    set_error("ql_ggml_dequant: ggml type %d has no native kernel (Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14)",
              ggml_type);
    return QL_ERR_UNSUPPORTED;
  }
  if (ggml_type == kQ4_K) return ql_q4k_dequant(raw, W, N, K, stream);
  if (!raw || !W || N <= 0 || K <= 0 || K % 256 != 0) {
    set_error("ql_ggml_dequant: bad arguments (N=%d K=%d; K a positive multiple of 256)", N, K);
    return QL_ERR_ARG;
  }
  const long nruns = (long)N * (K / 256);
  const long need = (nruns * 32 + 255) / 256;
  const unsigned grid = (unsigned)(need < 148 * 64 ? need : 148 * 64);
  cudaStream_t st = (cudaStream_t)stream;
  switch (ggml_type) {
    case kQ8_0: ggml_dequant_kernel<kQ8_0><<<grid, 256, 0, st>>>(raw, W, nruns); break;
    case kQ5_K: ggml_dequant_kernel<kQ5_K><<<grid, 256, 0, st>>>(raw, W, nruns); break;
    default: ggml_dequant_kernel<kQ6_K><<<grid, 256, 0, st>>>(raw, W, nruns); break;
  }
  return cuda_status(cudaGetLastError(), "ql_ggml_dequant launch");
}

extern "C" int ql_ggml_matmul(const void* x, int x_dtype, long ldx, const uint8_t* raw, int ggml_type,
                              const float* bias, void* out, int out_dtype, long ldo, int M, int K, int N,
                              void* stream) {
  int vals, bytes;
  if (!type_info(ggml_type, vals, bytes)) {
    set_error("ql_ggml_matmul: ggml type %d has no native kernel (Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14)",
              ggml_type);
    return QL_ERR_UNSUPPORTED;
  }
  if (ggml_type == kQ4_K) return ql_q4k_matmul(x, x_dtype, ldx, raw, bias, out, out_dtype, ldo, M, K, N, stream);
  if (x_dtype < QL_F32 || x_dtype > QL_BF16 || out_dtype < QL_F32 || out_dtype > QL_BF16) {
    set_error("ql_ggml_matmul: unknown dtype code");
    return QL_ERR_ARG;
  }
  if (M < 0 || N <= 0 || K <= 0 || K % 256 != 0 || ldx < K || ldo < N) {
    set_error("ql_ggml_matmul: bad sizes (M=%d N=%d K=%d; K a positive multiple of 256)", M, N, K);
    return QL_ERR_ARG;
  }
  if (M == 0) return QL_OK;
  if (!x || !raw || !out) {
    set_error("ql_ggml_matmul: null pointer");
    return QL_ERR_ARG;
  }
  const long row_bytes = (long)(K / vals) * bytes;
  if ((reinterpret_cast<uintptr_t>(raw) & 3) || (row_bytes & 3)) {
    set_error("ql_ggml_matmul: rows of %ld bytes at %p are not 4-byte aligned (Q6_K needs K %% 512 == 0, Q8_0 "
              "K %% 64 == 0)", row_bytes, (const void*)raw);
    return QL_ERR_ALIGN;
  }
  GemvArgs a;
  a.x = x; a.x_dtype = x_dtype; a.ldx = ldx; a.raw = raw; a.row_bytes = row_bytes; a.bias = bias;
  a.out = out; a.out_dtype = out_dtype; a.ldo = ldo; a.M = M; a.K = K; a.N = N;
  cudaStream_t st = (cudaStream_t)stream;
  switch (ggml_type) {
    case kQ8_0: return launch_gemv<kQ8_0>(a, st);
    case kQ5_K: return launch_gemv<kQ5_K>(a, st);
    default:
      if (K % 512 != 0) {
        set_error("ql_ggml_matmul: Q6_K needs K %% 512 == 0 (K=%d)", K);
        return QL_ERR_UNSUPPORTED;
      }
      return launch_gemv<kQ6_K>(a, st);
  }
}
