// GGUF Q4_K on B200: exact dequant and the decode GEMV/GEMM that reads the file's own
// super-block layout (no load-time re-layout).
//
// Reference semantics (webtorch/ggufload.py:120-131, 190-202): a row of the [N, K] weight is
// K/256 blocks of 144 bytes: f16 d | f16 dmin | scales[12] | qs[128]. Sub-block j (32 values)
// has 6-bit scale sc_j and min m_j (get_scale_min_k4); value = (d*sc_j) * q - dmin*m_j, with q
// the low nibbles of qs[32g .. 32g+31] for j = 2g and the high nibbles for j = 2g+1.
//
// The decode GEMV / small-M GEMM runs the TMA-fed integer-MMA kernel of q4k_gemv_tma.cu; the
// register-fed kernel below serves the calls that kernel declines (no tensor-map encoder, an
// activation slice too large for shared memory). Its design:
//  * A warp owns 16 output rows; lane (g = lane/4, t = lane%4) streams rows g and g+8. For
//    each 32-byte quant group of a block, lane t reads its 8 bytes of both rows, so every
//    warp load touches 8 rows x 32 contiguous bytes.
//  * Nibbles become fp16 "1024 + q" (low) or "1024 + 16 q" (high) with one LOP3 each and are
//    fed to mma.sync unchanged; the 1024 (and /16) offsets are folded into per-(row, sub-block)
//    coefficients applied to the fp32 partial sums:
//      low:  d*sc * C - (1024 d*sc + dmin*m) * sum(x_sub)
//      high: d*sc/16 * C - (64 d*sc + dmin*m) * sum(x_sub)
//  * The scale half (a * C) lives in the MMA fragment layout; the sum(x) half is accumulated
//    by a second lane mapping (one lane per row and half-block) so each term is computed once.
//  * x is staged per CTA as power-of-two-scaled fp16 (exact rescale) with per-sub-block sums;
//    split-K across a thread-block cluster, reduced through distributed shared memory.
#include <cooperative_groups.h>

#include "ql_common.cuh"

namespace cg = cooperative_groups;

namespace ql {
namespace {

constexpr int kBlkVals = 256;
constexpr int kBlkBytes = 144;

__device__ __forceinline__ float f16_bits_to_float(uint32_t h) {
  return __half2float(__ushort_as_half((unsigned short)(h & 0xffffu)));
}

__global__ void q4k_dequant_kernel(const uint8_t* __restrict__ raw, float* __restrict__ W, long nblocks) {
  // one thread per (block, 32-value sub-block)
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nblocks * 8; i += (long)gridDim.x * blockDim.x) {
    const long b = i >> 3;
    const int j = (int)(i & 7);
    const uint8_t* blk = raw + b * kBlkBytes;
    const uint32_t h0 = blk[0] | (blk[1] << 8), h1 = blk[2] | (blk[3] << 8);
    const uint32_t s0 = blk[4] | (blk[5] << 8) | (blk[6] << 16) | ((uint32_t)blk[7] << 24);
    const uint32_t s1 = blk[8] | (blk[9] << 8) | (blk[10] << 16) | ((uint32_t)blk[11] << 24);
    const uint32_t s2 = blk[12] | (blk[13] << 8) | (blk[14] << 16) | ((uint32_t)blk[15] << 24);
    uint32_t sc, m;
    q4k_scale_min(s0, s1, s2, j, sc, m);
    // numpy: d1 = d * sc (f32), m1 = dmin * m (f32), value = d1 * q - m1 (two roundings)
    const float d1 = __fmul_rn(f16_bits_to_float(h0), (float)sc);
    const float m1 = __fmul_rn(f16_bits_to_float(h1), (float)m);
    const uint8_t* qs = blk + 16 + 32 * (j >> 1);
    const int sh = (j & 1) ? 4 : 0;
    float* out = W + b * kBlkVals + j * 32;
    for (int l = 0; l < 32; ++l) out[l] = __fsub_rn(__fmul_rn(d1, (float)((qs[l] >> sh) & 15)), m1);
  }
}

constexpr int kNW = 4;              // warps per CTA
constexpr int kCtaRows = kNW * 16;  // output rows per CTA

struct Q4kArgs {
  const void* x;
  long ldx;
  int x_dtype;
  const uint8_t* raw;
  long rowbytes;
  const float* bias;
  void* out;
  long ldo;
  int out_dtype;
  int M, K, N;
  int nb;  // blocks per row
  int cs;  // cluster size along K
};

// Stage x[:, kb0*256 : kb1*256] as power-of-two-scaled fp16, each 4-value chunk stored in the
// order (0, 2, 1, 3) the nibble-pair unpack produces, plus fp32 sums per 32-value sub-block.
__device__ void q4k_stage_x(const Q4kArgs& a, int k0, int klen, int xsum_stride, __half* xs, float* xsum,
                            int* sh_exp, unsigned* sh_max) {
  const int tid = threadIdx.x, nthr = blockDim.x, M = a.M;
  if (tid < 16) sh_max[tid] = 0u;
  __syncthreads();
  for (int m = 0; m < M; ++m) {
    float mx = 0.f;
    for (int kk = tid; kk < klen; kk += nthr)
      mx = fmaxf(mx, fabsf(load_as_float(a.x, a.x_dtype, (long)m * a.ldx + k0 + kk)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) atomicMax(&sh_max[m], __float_as_uint(mx));
  }
  __syncthreads();
  if (tid < M) sh_exp[tid] = stage_exponent(__uint_as_float(sh_max[tid]));
  __syncthreads();
  // one 32-value sub-block per iteration: convert, permute, store, and sum the staged values
  const int nsub = klen / 32;
  for (int i = tid; i < M * nsub; i += nthr) {
    const int m = i / nsub, sb = i % nsub;
    const float s = exp2i(-sh_exp[m]);
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      __align__(8) __half v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __half h = __float2half_rn(load_as_float(a.x, a.x_dtype, (long)m * a.ldx + k0 + sb * 32 + c * 4 + e) * s);
        sum += __half2float(h);
        v[(e & 1) * 2 + (e >> 1)] = h;
      }
      *reinterpret_cast<uint2*>(xs + (long)m * klen + sb * 32 + c * 4) = *reinterpret_cast<uint2*>(v);
    }
    xsum[m * xsum_stride + sb] = sum;
  }
  __syncthreads();
}

template <int MT>
__global__ void __launch_bounds__(kNW * 32, 4) q4k_gemv_kernel(const Q4kArgs a) {
  constexpr int MAXM = 8 * MT;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int sh_exp[16];
  __shared__ unsigned sh_max[16];
  __shared__ float sh_corr[kNW][16][MAXM];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, t = lane & 3;
  const int rank = blockIdx.x;
  const int b0 = (int)((long)a.nb * rank / a.cs), b1 = (int)((long)a.nb * (rank + 1) / a.cs);
  const int nbl = b1 - b0;
  const int nb_max = (a.nb + a.cs - 1) / a.cs;
  const int k0 = b0 * kBlkVals, klen = nbl * kBlkVals;
  const int M = a.M, N = a.N;

  __half* xs = reinterpret_cast<__half*>(smem);
  const int xs_bytes = (M * nb_max * kBlkVals * 2 + 15) & ~15;
  float* xsum = reinterpret_cast<float*>(smem + xs_bytes);
  const int xsum_bytes = (M * nb_max * 8 * 4 + 15) & ~15;
  float* red = reinterpret_cast<float*>(smem + xs_bytes + xsum_bytes);  // [kCtaRows][MAXM]

  q4k_stage_x(a, k0, klen, nb_max * 8, xs, xsum, sh_exp, sh_max);

  const int rbase = blockIdx.y * kCtaRows + warp * 16;
  const int rA = rbase + gq, rB = rbase + gq + 8;   // MMA-layout rows
  const bool okA = rA < N, okB = rB < N;
  const uint8_t* pA = a.raw + (long)(okA ? rA : 0) * a.rowbytes;
  const uint8_t* pB = a.raw + (long)(okB ? rB : 0) * a.rowbytes;
  const int rC = rbase + (lane & 15);               // correction-layout row
  const bool okC = rC < N;
  const uint8_t* pC = a.raw + (long)(okC ? rC : 0) * a.rowbytes;
  const int jhalf = lane >> 4;                      // sub-blocks 4*jhalf .. 4*jhalf+3

  float acc[MT][4];
  float corr[MAXM];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[mt][i] = 0.f;
#pragma unroll
  for (int m = 0; m < MAXM; ++m) corr[m] = 0.f;

  for (int bl = 0; bl < nbl; ++bl) {
    const long boff = (long)(b0 + bl) * kBlkBytes;
    // ---- loads: headers of rows A, B, C and this lane's 8 bytes of each quant group of A and B
    const uint4 hA = okA ? ldg_stream_v4(pA + boff) : make_uint4(0, 0, 0, 0);
    const uint4 hB = okB ? ldg_stream_v4(pB + boff) : make_uint4(0, 0, 0, 0);
    const uint4 hC = okC ? *reinterpret_cast<const uint4*>(pC + boff) : make_uint4(0, 0, 0, 0);
    uint2 qA[4], qB[4];
#pragma unroll
    for (int G = 0; G < 4; ++G) {
      qA[G] = okA ? ldg_stream_v2(pA + boff + 16 + 32 * G + 8 * t) : make_uint2(0, 0);
      qB[G] = okB ? ldg_stream_v2(pB + boff + 16 + 32 * G + 8 * t) : make_uint2(0, 0);
    }
    // ---- per-lane decode of d*sc for sub-blocks 2t, 2t+1 of rows A and B (shared by shuffles)
    float dscA[2], dscB[2];
    {
      const float dA = f16_bits_to_float(hA.x), dB = f16_bits_to_float(hB.x);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        uint32_t sc, m;
        q4k_scale_min(hA.y, hA.z, hA.w, 2 * t + u, sc, m);
        dscA[u] = dA * (float)sc;
        q4k_scale_min(hB.y, hB.z, hB.w, 2 * t + u, sc, m);
        dscB[u] = dB * (float)sc;
      }
    }
    // ---- correction lanes: (1024 | 64) * d*sc + dmin*m times the staged sub-block sums
    {
      const float d = f16_bits_to_float(hC.x), dmin = f16_bits_to_float(hC.x >> 16);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = 4 * jhalf + u;
        uint32_t sc, m;
        q4k_scale_min(hC.y, hC.z, hC.w, j, sc, m);
        const float coef = ((j & 1) ? 64.f : 1024.f) * (d * (float)sc) + dmin * (float)m;
#pragma unroll
        for (int tok = 0; tok < MAXM; ++tok)
          if (tok < M) corr[tok] = fmaf(coef, xsum[tok * (nb_max * 8) + bl * 8 + j], corr[tok]);
      }
    }
    // ---- tensor-core partial sums, one 32-byte quant group (two sub-blocks) at a time
#pragma unroll
    for (int G = 0; G < 4; ++G) {
      const float aA_lo = __shfl_sync(0xffffffffu, dscA[0], gq * 4 + G);
      const float aA_hi = __shfl_sync(0xffffffffu, dscA[1], gq * 4 + G) * 0.0625f;
      const float aB_lo = __shfl_sync(0xffffffffu, dscB[0], gq * 4 + G);
      const float aB_hi = __shfl_sync(0xffffffffu, dscB[1], gq * 4 + G) * 0.0625f;
      uint32_t loA[2][2], hiA[2][2], loB[2][2], hiB[2][2];
      const uint32_t wA[2] = {qA[G].x, qA[G].y}, wB[2] = {qB[G].x, qB[G].y};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        loA[h][0] = lop3_andor(wA[h], 0x000F000Fu, kMagicF16x2);
        hiA[h][0] = lop3_andor(wA[h], 0x00F000F0u, kMagicF16x2);
        loA[h][1] = lop3_andor(wA[h] >> 8, 0x000F000Fu, kMagicF16x2);
        hiA[h][1] = lop3_andor(wA[h] >> 8, 0x00F000F0u, kMagicF16x2);
        loB[h][0] = lop3_andor(wB[h], 0x000F000Fu, kMagicF16x2);
        hiB[h][0] = lop3_andor(wB[h], 0x00F000F0u, kMagicF16x2);
        loB[h][1] = lop3_andor(wB[h] >> 8, 0x000F000Fu, kMagicF16x2);
        hiB[h][1] = lop3_andor(wB[h] >> 8, 0x00F000F0u, kMagicF16x2);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int tok = gq + 8 * mt;
        float clo[4] = {0.f, 0.f, 0.f, 0.f}, chi[4] = {0.f, 0.f, 0.f, 0.f};
        uint4 xlo = make_uint4(0, 0, 0, 0), xhi = make_uint4(0, 0, 0, 0);
        if (tok < M) {
          const __half* xr = xs + (long)tok * klen + bl * kBlkVals + 8 * t;
          xlo = *reinterpret_cast<const uint4*>(xr + (2 * G) * 32);
          xhi = *reinterpret_cast<const uint4*>(xr + (2 * G + 1) * 32);
        }
        mma_16816_f16(clo, loA[0][0], loB[0][0], loA[0][1], loB[0][1], xlo.x, xlo.y);
        mma_16816_f16(clo, loA[1][0], loB[1][0], loA[1][1], loB[1][1], xlo.z, xlo.w);
        mma_16816_f16(chi, hiA[0][0], hiB[0][0], hiA[0][1], hiB[0][1], xhi.x, xhi.y);
        mma_16816_f16(chi, hiA[1][0], hiB[1][0], hiA[1][1], hiB[1][1], xhi.z, xhi.w);
        acc[mt][0] = fmaf(aA_lo, clo[0], fmaf(aA_hi, chi[0], acc[mt][0]));
        acc[mt][1] = fmaf(aA_lo, clo[1], fmaf(aA_hi, chi[1], acc[mt][1]));
        acc[mt][2] = fmaf(aB_lo, clo[2], fmaf(aB_hi, chi[2], acc[mt][2]));
        acc[mt][3] = fmaf(aB_lo, clo[3], fmaf(aB_hi, chi[3], acc[mt][3]));
      }
    }
  }

  // ---- combine the two halves of the correction (lanes r and r+16 hold row r) in smem
#pragma unroll
  for (int tok = 0; tok < MAXM; ++tok) corr[tok] += __shfl_xor_sync(0xffffffffu, corr[tok], 16);
  if (lane < 16) {
#pragma unroll
    for (int tok = 0; tok < MAXM; ++tok) sh_corr[warp][lane][tok] = corr[tok];
  }
  __syncwarp();

  // C fragment: [0],[1] -> row gq, tokens 2t, 2t+1; [2],[3] -> row gq+8
  if (a.cs == 1) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tok = 8 * mt + 2 * t + (i & 1);
        const int lr = gq + 8 * (i >> 1);
        const int row = rbase + lr;
        if (tok < M && row < N) {
          float v = (acc[mt][i] - sh_corr[warp][lr][tok]) * exp2i(sh_exp[tok]);
          if (a.bias) v += a.bias[row];
          store_from_float(a.out, a.out_dtype, (long)tok * a.ldo + row, v);
        }
      }
    return;
  }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tok = 8 * mt + 2 * t + (i & 1);
      const int lr = gq + 8 * (i >> 1);
      if (tok < M) red[(warp * 16 + lr) * MAXM + tok] = (acc[mt][i] - sh_corr[warp][lr][tok]) * exp2i(sh_exp[tok]);
    }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const int total = kCtaRows * M;
  const int lo = (int)((long)total * rank / a.cs), hi = (int)((long)total * (rank + 1) / a.cs);
  for (int idx = lo + tid; idx < hi; idx += blockDim.x) {
    const int lrow = idx / M, tok = idx % M;
    const int row = blockIdx.y * kCtaRows + lrow;
    float v = 0.f;
    for (int q = 0; q < a.cs; ++q) v += cluster.map_shared_rank(red, q)[lrow * MAXM + tok];
    if (row < N) {
      if (a.bias) v += a.bias[row];
      store_from_float(a.out, a.out_dtype, (long)tok * a.ldo + row, v);
    }
  }
  cluster.sync();
}

template <int MT>
int launch_q4k(const Q4kArgs& a, cudaStream_t st) {
  auto kern = q4k_gemv_kernel<MT>;
  const int nb_max = (a.nb + a.cs - 1) / a.cs;
  const size_t xs_bytes = ((size_t)a.M * nb_max * kBlkVals * 2 + 15) & ~(size_t)15;
  const size_t xsum_bytes = ((size_t)a.M * nb_max * 8 * 4 + 15) & ~(size_t)15;
  const size_t smem = xs_bytes + xsum_bytes + (size_t)kCtaRows * 8 * MT * 4;
  if (smem > 180 * 1024) {
    set_error("ql_q4k_matmul: activation slice needs %zu bytes of shared memory (M=%d, K=%d)", smem, a.M, a.K);
    return QL_ERR_UNSUPPORTED;
  }
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 180 * 1024),
                         "cudaFuncSetAttribute(smem)");
    if (rc) return rc;
    rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                     "cudaFuncSetAttribute(cluster)");
    if (rc) return rc;
    configured_dev = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.cs, (a.N + kCtaRows - 1) / kCtaRows, 1);
  cfg.blockDim = dim3(kNW * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, a), "q4k_gemv launch");
}

inline int pow2_floor(int v) {
  int p = 1;
  while (p * 2 <= v) p *= 2;
  return p;
}

int q4k_gemv(const void* x, int x_dtype, long ldx, const uint8_t* raw, const float* bias, void* out, int out_dtype,
             long ldo, int M, int K, int N, cudaStream_t st) {
  Q4kArgs a;
  a.x = x; a.ldx = ldx; a.x_dtype = x_dtype; a.raw = raw;
  a.nb = K / kBlkVals;
  a.rowbytes = (long)a.nb * kBlkBytes;
  a.bias = bias; a.out = out; a.ldo = ldo; a.out_dtype = out_dtype;
  a.M = M; a.K = K; a.N = N;
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int cta_rows = (N + kCtaRows - 1) / kCtaRows;
  int cs = pow2_floor(sms * 4 / cta_rows > 0 ? sms * 4 / cta_rows : 1);
  if (cs > 16) cs = 16;
  while (cs > 1 && cs > a.nb) cs /= 2;
  while (cs < 16 && cs < a.nb && (size_t)M * ((a.nb + cs - 1) / cs) * kBlkVals * 2 > 96 * 1024) cs *= 2;
  a.cs = cs;
  return M <= 8 ? launch_q4k<1>(a, st) : launch_q4k<2>(a, st);
}

}  // namespace
}  // namespace ql

namespace ql {
bool q4k_gemv_tma(const void* x, int x_dtype, long ldx, const uint8_t* raw, const float* bias, void* out,
                  int out_dtype, long ldo, int M, int K, int N, cudaStream_t st, int* rc, void* workspace,
                  size_t ws_bytes);
size_t q4k_stage_workspace(int M, int K);
int q4k_gemm_sm100(const void* x, int x_dtype, long ldx, const uint8_t* raw, const float* bias, void* out,
                   int out_dtype, long ldo, int M, int K, int N, void* workspace, size_t ws_bytes, cudaStream_t st,
                   bool* handled);
size_t gptq_gemm_workspace(int M, int K);
int q4k_gemm_min_m();
}

using namespace ql;

extern "C" int ql_q4k_dequant(const uint8_t* raw, float* W, int N, int K, void* stream) {
  if (!raw || !W || N <= 0 || K <= 0 || K % kBlkVals != 0) {
    set_error("ql_q4k_dequant: bad arguments (N=%d K=%d; K must be a positive multiple of 256)", N, K);
    return QL_ERR_ARG;
  }
  const long nblocks = (long)N * (K / kBlkVals);
  const long threads = 256, need = (nblocks * 8 + threads - 1) / threads;
  q4k_dequant_kernel<<<(unsigned)(need < 148 * 32 ? need : 148 * 32), threads, 0, (cudaStream_t)stream>>>(raw, W, nblocks);
  return cuda_status(cudaGetLastError(), "ql_q4k_dequant launch");
}

static int q4k_matmul_impl(const void* x, int x_dtype, long ldx, const uint8_t* raw, const float* bias, void* out,
                           int out_dtype, long ldo, int M, int K, int N, void* workspace, size_t ws_bytes,
                           void* stream) {
  if (x_dtype < QL_F32 || x_dtype > QL_BF16 || out_dtype < QL_F32 || out_dtype > QL_BF16) {
    set_error("ql_q4k_matmul: unknown dtype code");
    return QL_ERR_ARG;
  }
  if (M < 0 || N <= 0 || K <= 0 || K % kBlkVals != 0) {
    set_error("ql_q4k_matmul: bad sizes (M=%d N=%d K=%d; K must be a positive multiple of 256)", M, N, K);
    return QL_ERR_ARG;
  }
  if (M == 0) return QL_OK;
  if (!x || !raw || !out || ldx < K || ldo < N) {
    set_error("ql_q4k_matmul: null pointer or short row stride");
    return QL_ERR_ARG;
  }
  if ((reinterpret_cast<uintptr_t>(raw) & 15) != 0) {
    set_error("ql_q4k_matmul: the raw Q4_K buffer must be 16-byte aligned");
    return QL_ERR_ALIGN;
  }
  cudaStream_t st = (cudaStream_t)stream;
  int rc = QL_OK;
  bool handled = false;
  rc = q4k_gemm_sm100(x, x_dtype, ldx, raw, bias, out, out_dtype, ldo, M, K, N, workspace, ws_bytes, st, &handled);
  if (handled) return rc;
  if (q4k_gemv_tma(x, x_dtype, ldx, raw, bias, out, out_dtype, ldo, M, K, N, st, &rc, workspace, ws_bytes)) return rc;
  for (int m0 = 0; m0 < M; m0 += 16) {
    const int mc = (M - m0) < 16 ? (M - m0) : 16;
    const char* xb = reinterpret_cast<const char*>(x) + (long)m0 * ldx * (x_dtype == QL_F32 ? 4 : 2);
    char* ob = reinterpret_cast<char*>(out) + (long)m0 * ldo * (out_dtype == QL_F32 ? 4 : 2);
    const int rc = q4k_gemv(xb, x_dtype, ldx, raw, bias, ob, out_dtype, ldo, mc, K, N, st);
    if (rc) return rc;
  }
  return QL_OK;
}

extern "C" int ql_q4k_matmul(const void* x, int x_dtype, long ldx, const uint8_t* raw, const float* bias, void* out,
                             int out_dtype, long ldo, int M, int K, int N, void* stream) {
  return q4k_matmul_impl(x, x_dtype, ldx, raw, bias, out, out_dtype, ldo, M, K, N, nullptr, 0, stream);
}

extern "C" size_t ql_q4k_matmul_workspace(int M, int K) {
  if (M <= 0 || K <= 0 || K % kBlkVals != 0) return 0;
  const size_t a = q4k_stage_workspace(M, K);                                  // decode path
  const size_t b = M >= q4k_gemm_min_m() ? gptq_gemm_workspace(M, K) : 0;     // tensor-core path
  return a > b ? a : b;
}

extern "C" int ql_q4k_matmul_ws(const void* x, int x_dtype, long ldx, const uint8_t* raw, const float* bias,
                                void* out, int out_dtype, long ldo, int M, int K, int N, void* workspace,
                                size_t workspace_bytes, void* stream) {
  return q4k_matmul_impl(x, x_dtype, ldx, raw, bias, out, out_dtype, ldo, M, K, N, workspace, workspace_bytes, stream);
}
