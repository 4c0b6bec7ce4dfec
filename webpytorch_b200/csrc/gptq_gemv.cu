// GPTQ int4/int8 quantized linear on B200: exact dequant, act-order row sort, and the
// decode GEMV (small M) that streams packed weights at HBM speed.
//
// Reference semantics (webtorch/_core.py:4046-4072, _gptq_matmul_np):
//   q[k, n]  = (qweight[k / per, n] >> (bits * (k % per))) & (2^bits - 1)
//   z[g, n]  = (qzeros[g, n / per] >> (bits * (n % per))) & (2^bits - 1)
//   W[k, n]  = scales[g, n] * (q[k, n] - (z[g, n] + zero_offset)),  g = k / gs
//   y        = x @ W (+ bias)
//
// GEMV design (decode, M <= 16 per launch):
//  * A warp owns a strip of 32 output columns. Lane (gq = lane/4, t = lane%4) streams one
//    16-byte vector per step: 4 adjacent columns of packed row 4*step + t. A warp load is
//    therefore 4 rows x 128 contiguous bytes, fully used.
//  * Nibbles (or bytes) become fp16 integers with one LOP3 each (magic 0x6400 = 1024.0),
//    and the zero point (z + zero_offset) is removed with one HSUB2/HFMA2, so q - z - off
//    is exact in fp16.
//  * The dot product and the 4-lane K reduction run on the tensor cores with register
//    operands (mma.sync m16n8k16): the MMA's 16 rows are the lane-quads' columns, its 8
//    columns are tokens. Register operands keep the dequantised weights out of shared
//    memory, which a bandwidth-bound GEMV cannot afford to write and re-read.
//  * Each group's partial sum is scaled in fp32 (acc += scale * partial), so the only
//    roundings are the fp16 staging of x (power-of-two scaled per row, see below) and the
//    fp32 accumulation.
//  * Split-K runs across a thread-block cluster; partial sums are reduced through
//    distributed shared memory in a fixed order (deterministic, no scratch, no atomics).
//  * Activations are staged once per CTA into shared memory as fp16, each token row scaled
//    by an exact power of two so its largest value sits in [2^14, 2^15); the scale is undone
//    on the partial sums. The staging also applies the act-order gather x[:, perm[k]].
#include <cooperative_groups.h>

#include "ql_common.cuh"
#include "gemv_common.cuh"

namespace cg = cooperative_groups;
using ql::gemv::chunk_pos;

namespace ql {
namespace {

// ---------------------------------------------------------------------------------------
// exact dequant (test oracle partner and load-time helper)
// ---------------------------------------------------------------------------------------
__global__ void gptq_dequant_kernel(const uint32_t* __restrict__ qw, const uint32_t* __restrict__ qz,
                                    const void* __restrict__ sc, int sc_dtype,
                                    const int32_t* __restrict__ g_idx, float* __restrict__ W, int K,
                                    int N, int gs, int bits, double zoff) {
  const int per = 32 / bits;
  const uint32_t mask = (1u << bits) - 1u;
  const long total = (long)(K / per) * N;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total;
       i += (long)gridDim.x * blockDim.x) {
    const int n = (int)(i % N);
    const int r = (int)(i / N);
    const uint32_t w = qw[i];
    for (int j = 0; j < per; ++j) {
      const int k = r * per + j;
      const int g = g_idx ? g_idx[k] : k / gs;
      const uint32_t q = (w >> (bits * j)) & mask;
      const uint32_t z = (qz[(long)g * (N / per) + n / per] >> (bits * (n % per))) & mask;
      const double s = (double)load_as_float(sc, sc_dtype, (long)g * N + n);
      // numpy: float32 scale * float64 (q - (z + zoff)), then one rounding to float32
      W[(long)k * N + n] = __double2float_rn(s * ((double)q - ((double)z + zoff)));
    }
  }
}

__global__ void gptq_sort_rows_kernel(const uint32_t* __restrict__ qin, const int32_t* __restrict__ perm,
                                      uint32_t* __restrict__ qout, int K, int N, int bits) {
  const int per = 32 / bits;
  const uint32_t mask = (1u << bits) - 1u;
  const long total = (long)(K / per) * N;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total;
       i += (long)gridDim.x * blockDim.x) {
    const int n = (int)(i % N);
    const int r = (int)(i / N);
    uint32_t acc = 0;
    for (int j = 0; j < per; ++j) {
      const int src = perm[r * per + j];
      const uint32_t q = (qin[(long)(src / per) * N + n] >> (bits * (src % per))) & mask;
      acc |= q << (bits * j);
    }
    qout[i] = acc;
  }
}

// ---------------------------------------------------------------------------------------
// decode GEMV
// ---------------------------------------------------------------------------------------
constexpr int kNW = 4;           // warps per CTA, one 32-column strip each
constexpr int kCtaCols = kNW * 32;

struct GemvArgs {
  const void* x;
  const int32_t* x_rows;   // NULL, or token row of x for each staged row (MoE gather)
  const int32_t* x_perm;
  long ldx;
  int x_dtype;
  int x_vec;    // x rows may be read with 16-byte vector loads
  const uint32_t* qw;
  const uint32_t* qz;
  const void* sc;
  int sc_dtype;
  const float* bias;
  void* out;
  long ldo;
  int out_dtype;
  int M, K, N;
  int G;        // number of GS-row kernel groups (K / GS)
  int gs_mult;  // scale/zero row = kernel group / gs_mult (checkpoint group size = GS * gs_mult)
  int lg_gs_mult;  // log2(gs_mult) when it is a power of two, else -1
  int cs;       // cluster size along K (== gridDim.x), a power of two
  int lg_cs;
  float zoff;
  // grouped (MoE) mode, when moe_offsets != NULL: blockIdx.z picks an active expert, whose
  // rows [offsets[e], offsets[e + 1]) of x/out are processed in chunks of 8 * MT
  const int32_t* moe_offsets;
  const int32_t* moe_active;
  const int32_t* moe_n_active;
  long qw_estride, qz_estride, sc_estride;   // elements between consecutive experts
  int glu;   // > 0: x rows are [gate | up] glu elements apart (SwiGLU applied when staging)
  const float* nw = nullptr;   // RMSNorm folded into the loads: not used by this kernel
  const float* nr = nullptr;
};

// Register-resident batch of UG consecutive groups of one lane's weights, scales and zeros.
template <int BITS, int GS>
struct WBatch {
  static constexpr int PER = 32 / BITS;
  static constexpr int SPG = GS / (4 * PER);           // 16-byte loads per lane per group
  static constexpr int UG = SPG >= 4 ? 1 : 4 / SPG;   // groups per batch (>= 4 loads in flight)
  uint4 w[UG][SPG];
  float sc[UG][4];
  uint32_t z[UG];
};

template <int BITS, int GS>
__device__ __forceinline__ void load_batch(WBatch<BITS, GS>& B, const GemvArgs& a, int grp0, int gend, int c0,
                                           bool col_ok, int t) {
  using W = WBatch<BITS, GS>;
  const int N = a.N;
#pragma unroll
  for (int u = 0; u < W::UG; ++u) {
    const int grp = grp0 + u;
    const bool ok = col_ok && grp < gend;
    const int srow = a.lg_gs_mult >= 0 ? (grp >> a.lg_gs_mult) : grp / a.gs_mult;
    const uint32_t* wp = a.qw + (size_t)(grp * (GS / W::PER) + t) * N + c0;
#pragma unroll
    for (int s = 0; s < W::SPG; ++s) {
      B.w[u][s] = ok ? ldg_stream_v4(wp + (size_t)(s * 4) * N) : make_uint4(0, 0, 0, 0);
    }
    if (ok) {
      if (a.sc_dtype == QL_F16) {
        const uint2 h = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(a.sc) + (long)srow * N + c0);
        const float2 f0 = __half22float2(u32_as_h2(h.x));
        const float2 f1 = __half22float2(u32_as_h2(h.y));
        B.sc[u][0] = f0.x; B.sc[u][1] = f0.y; B.sc[u][2] = f1.x; B.sc[u][3] = f1.y;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) B.sc[u][i] = load_as_float(a.sc, a.sc_dtype, (long)srow * N + c0 + i);
      }
      B.z[u] = a.qz[(long)srow * (N / W::PER) + c0 / W::PER] >> (BITS * (c0 % W::PER));
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) B.sc[u][i] = 0.f;
      B.z[u] = 0;
    }
  }
}

// Multiply-accumulate one batch; g_local0 = index of its first group inside the staged slice.
template <int BITS, int GS, int MT>
__device__ __forceinline__ void compute_batch(const WBatch<BITS, GS>& B, float (&acc)[2][MT][4], const __half* xs,
                                              const float2* gsum, int gstride, int klen, int g_local0, int nvalid,
                                              int gq, int t, int M, float zoff) {
  using W = WBatch<BITS, GS>;
  constexpr uint32_t MASK = (1u << BITS) - 1u;
#pragma unroll
  for (int u = 0; u < W::UG; ++u) {
    if (u >= nvalid) break;  // warp-uniform
    const int gl = g_local0 + u;
    float gacc[2][MT][4];
#pragma unroll
    for (int p = 0; p < 2; ++p)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) gacc[p][mt][i] = 0.f;
#pragma unroll
    for (int s = 0; s < W::SPG; ++s) {
      const int koff = gl * GS + (s * 4 + t) * W::PER;
      const uint32_t wcol[4] = {B.w[u][s].x, B.w[u][s].y, B.w[u][s].z, B.w[u][s].w};
      if constexpr (BITS == 4) {
        uint32_t P[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t w8 = wcol[i] >> 8;
          P[i][0] = lop3_andor(wcol[i], 0x000F000Fu, kMagicF16x2);   // 1024 + q0 | 1024 + q4
          P[i][1] = lop3_andor(wcol[i], 0x00F000F0u, kMagicF16x2);   // 1024 + 16 q1 | 1024 + 16 q5
          P[i][2] = lop3_andor(w8, 0x000F000Fu, kMagicF16x2);        // q2 | q6
          P[i][3] = lop3_andor(w8, 0x00F000F0u, kMagicF16x2);        // 16 q3 | 16 q7
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int tok = gq + 8 * mt;
          uint4 xv = make_uint4(0, 0, 0, 0);
          if (tok < M) xv = *reinterpret_cast<const uint4*>(xs + (long)tok * klen + koff);
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            mma_16816_f16(gacc[p][mt], P[2 * p][0], P[2 * p + 1][0], P[2 * p][1], P[2 * p + 1][1], xv.x, xv.y);
            mma_16816_f16(gacc[p][mt], P[2 * p][2], P[2 * p + 1][2], P[2 * p][3], P[2 * p + 1][3], xv.z, xv.w);
          }
        }
      } else {
        uint32_t P[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          P[i][0] = lop3_andor(wcol[i], 0x00FF00FFu, kMagicF16x2);      // 1024 + b0 | 1024 + b2
          P[i][1] = lop3_andor(wcol[i] >> 8, 0x00FF00FFu, kMagicF16x2); // 1024 + b1 | 1024 + b3
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int tok = gq + 8 * mt;
          uint2 xv = make_uint2(0, 0);
          if (tok < M) xv = *reinterpret_cast<const uint2*>(xs + (long)tok * klen + koff);
#pragma unroll
          for (int p = 0; p < 2; ++p)
            mma_16816_f16(gacc[p][mt], P[2 * p][0], P[2 * p + 1][0], P[2 * p][1], P[2 * p + 1][1], xv.x, xv.y);
        }
      }
    }
    // fold the magic offset and the zero point, then scale:
    //   acc += sc * (C - (1024 * A + (z + off) * S))
    float zc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) zc[i] = (float)((B.z[u] >> (BITS * i)) & MASK) + zoff;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      float A[2], S[2];
#pragma unroll
      for (int tk = 0; tk < 2; ++tk) {
        const int tok = 8 * mt + 2 * t + tk;
        const float2 as = tok < M ? gsum[tok * gstride + gl] : make_float2(0.f, 0.f);
        A[tk] = 1024.f * as.x;
        S[tk] = as.y;
      }
#pragma unroll
      for (int p = 0; p < 2; ++p)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int col = 2 * p + (i >> 1), tk = i & 1;
          const float v = gacc[p][mt][i] - fmaf(zc[col], S[tk], A[tk]);
          acc[p][mt][i] = fmaf(B.sc[u][col], v, acc[p][mt][i]);
        }
    }
  }
}

template <int BITS, int GS, int MT>
__device__ __forceinline__ void gemv_body(const GemvArgs& a);

template <int BITS, int GS, int MT, bool GROUPED>
__global__ void __launch_bounds__(kNW * 32, 4) gptq_gemv_kernel(const GemvArgs a) {
  if constexpr (!GROUPED) {
    gemv_body<BITS, GS, MT>(a);
    return;
  }
  // grouped experts: every CTA of a cluster shares blockIdx.z, so these exits are cluster-uniform
  const int slot = blockIdx.z;
  if (slot >= *a.moe_n_active) return;
  const int e = a.moe_active[slot];
  const int r0 = a.moe_offsets[e];
  const int ne = a.moe_offsets[e + 1] - r0;
  const int xsz = a.x_dtype == QL_F32 ? 4 : 2, osz = a.out_dtype == QL_F32 ? 4 : 2;
  const int ssz = a.sc_dtype == QL_F32 ? 4 : 2;
  GemvArgs c = a;
  c.qw = a.qw + (size_t)e * a.qw_estride;
  c.qz = a.qz + (size_t)e * a.qz_estride;
  c.sc = reinterpret_cast<const char*>(a.sc) + (size_t)e * a.sc_estride * ssz;
  for (int m0 = 0; m0 < ne; m0 += 8 * MT) {
    c.M = min(8 * MT, ne - m0);
    if (a.x_rows) {
      c.x_rows = a.x_rows + r0 + m0;
    } else {
      c.x = reinterpret_cast<const char*>(a.x) + (size_t)(r0 + m0) * a.ldx * xsz;
    }
    c.out = reinterpret_cast<char*>(a.out) + (size_t)(r0 + m0) * a.ldo * osz;
    gemv_body<BITS, GS, MT>(c);
  }
}

template <int BITS, int GS, int MT>
__device__ __forceinline__ void gemv_body(const GemvArgs& a) {
  using W = WBatch<BITS, GS>;
  constexpr int UG = W::UG;
  constexpr int MAXM = 8 * MT;

  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int sh_exp[16];
  __shared__ unsigned sh_max[16];

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, t = lane & 3;
  const int rank = blockIdx.x;  // position along K inside the cluster
  // balanced split of G groups over cs ranks: the first G % cs ranks take one extra group
  const int gq_base = a.G >> a.lg_cs, grem = a.G & (a.cs - 1);
  const int g0 = rank * gq_base + min(rank, grem);
  const int g1 = g0 + gq_base + (rank < grem ? 1 : 0);
  const int ng = g1 - g0;
  const int klen = ng * GS;
  const int M = a.M, N = a.N;
  const int c0 = blockIdx.y * kCtaCols + warp * 32 + gq * 4;
  const bool col_ok = c0 < N;

  if (a.cs > 1) cluster_arrive_relaxed();  // every CTA of the cluster is running before DSMEM use
  if (tid < 16) sh_max[tid] = 0u;

  // The first batch of weights is requested before anything else: it does not depend on
  // the previous kernel's results, so under PDL it streams while that kernel finishes.
  W A, B;
  load_batch<BITS, GS>(A, a, g0, g1, c0, col_ok, t);
  pdl_trigger();
  pdl_wait();

  // shared memory: staged x [M][klen_max] | group sums [M][ng_max] | partial sums
  // (offsets are the same in every CTA of the cluster: DSMEM maps a local address to the
  // same offset in the peer)
  const int ng_max = (a.G + a.cs - 1) / a.cs;
  const int klen_max = ng_max * GS;
  __half* xs = reinterpret_cast<__half*>(smem);
  const int xs_bytes = ((M * klen_max * 2) + 15) & ~15;
  float2* gsum = reinterpret_cast<float2*>(smem + xs_bytes);
  const int gs_bytes = ((M * ng_max * 8) + 15) & ~15;
  float* red = reinterpret_cast<float*>(smem + xs_bytes + gs_bytes);
  __syncthreads();  // sh_max zeroed
  gemv::stage_x<BITS, GS, false>(a, g0 * GS, klen, ng_max, xs, gsum, sh_exp, sh_max, tid, (int)blockDim.x);

  float acc[2][MT][4];
#pragma unroll
  for (int p = 0; p < 2; ++p)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[p][mt][i] = 0.f;

  // double-buffered batches: the next batch is in flight while the current one is consumed
  const int nbatch = (ng + UG - 1) / UG;
  for (int b = 0; b < nbatch; b += 2) {
    if (b + 1 < nbatch) load_batch<BITS, GS>(B, a, g0 + (b + 1) * UG, g1, c0, col_ok, t);
    compute_batch<BITS, GS, MT>(A, acc, xs, gsum, ng_max, klen, b * UG, ng - b * UG, gq, t, M, a.zoff);
    if (b + 2 < nbatch) load_batch<BITS, GS>(A, a, g0 + (b + 2) * UG, g1, c0, col_ok, t);
    if (b + 1 < nbatch)
      compute_batch<BITS, GS, MT>(B, acc, xs, gsum, ng_max, klen, (b + 1) * UG, ng - (b + 1) * UG, gq, t, M, a.zoff);
  }

  // ---- epilogue: undo the activation scale, then write (single CTA) or reduce (cluster)
  if (a.cs == 1) {
#pragma unroll
    for (int p = 0; p < 2; ++p)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tok = 8 * mt + 2 * t + (i & 1);
          const int col = c0 + 2 * p + (i >> 1);
          if (tok < M && col_ok) {
            float v = acc[p][mt][i] * exp2i(sh_exp[tok]);
            if (a.bias) v += a.bias[col];
            store_from_float(a.out, a.out_dtype, (long)tok * a.ldo + col, v);
          }
        }
    return;
  }

  // rank q owns CTA columns [q * cpo, (q + 1) * cpo), cpo = 128 / cs (cs is a power of two);
  // every CTA pushes its partials into the owner's shared memory, one cluster barrier
  // publishes them, and each owner sums its share in rank order
  cg::cluster_group cluster = cg::this_cluster();
  const int lg_cpo = 7 - (31 - __clz(a.cs));
  const int chunk = (kCtaCols >> (31 - __clz(a.cs))) * MAXM;   // floats per source rank
  float* mine[2];
  cluster_wait_acquire();  // pairs with the relaxed arrive at kernel start
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int lcol = warp * 32 + gq * 4 + 2 * p;    // columns lcol and lcol + 1 (same owner)
    const int owner = lcol >> lg_cpo;
    mine[p] = cluster.map_shared_rank(red, owner) + rank * chunk + (lcol - (owner << lg_cpo)) * MAXM;
  }
#pragma unroll
  for (int p = 0; p < 2; ++p)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tok = 8 * mt + 2 * t + (i & 1);
        if (tok < M) mine[p][(i >> 1) * MAXM + tok] = acc[p][mt][i] * exp2i(sh_exp[tok]);
      }
  cluster_arrive_release();
  cluster_wait_acquire();
  const int cpo = kCtaCols >> (31 - __clz(a.cs));
  for (int s = tid; s < cpo * M; s += blockDim.x) {
    const int c = s / M, tok = s - c * M;
    float v = 0.f;
    for (int q = 0; q < a.cs; ++q) v += red[q * chunk + c * MAXM + tok];
    const int col = blockIdx.y * kCtaCols + rank * cpo + c;
    if (col < N) {
      if (a.bias) v += a.bias[col];
      store_from_float(a.out, a.out_dtype, (long)tok * a.ldo + col, v);
    }
  }
}

template <int BITS, int GS, int MT, bool GROUPED>
int launch_gemv(const GemvArgs& a, cudaStream_t st, int zdim) {
  auto kern = gptq_gemv_kernel<BITS, GS, MT, GROUPED>;
  const int ng_max = (a.G + a.cs - 1) / a.cs;
  const size_t xs_bytes = ((size_t)a.M * ng_max * GS * 2 + 15) & ~(size_t)15;
  const size_t gs_bytes = ((size_t)a.M * ng_max * 8 + 15) & ~(size_t)15;
  const size_t smem = xs_bytes + gs_bytes + (size_t)kCtaCols * 8 * MT * sizeof(float);
  if (smem > 200 * 1024) {
    set_error("ql_gptq_matmul: activation slice needs %zu bytes of shared memory (M=%d, K=%d)", smem, a.M, a.K);
    return QL_ERR_UNSUPPORTED;
  }
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024),
                         "cudaFuncSetAttribute(smem)");
    if (rc) return rc;
    rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                     "cudaFuncSetAttribute(cluster)");
    if (rc) return rc;
    configured_dev = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.cs, (a.N + kCtaCols - 1) / kCtaCols, zdim);
  cfg.blockDim = dim3(kNW * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  int nattr = 1;
  if (launch_flags() & QL_LAUNCH_PDL) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    nattr = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, a), "gptq_gemv launch");
}

template <int BITS, int GS>
int dispatch_mt(const GemvArgs& a, cudaStream_t st, int zdim) {
  if (a.moe_offsets)
    return a.M <= 8 ? launch_gemv<BITS, GS, 1, true>(a, st, zdim) : launch_gemv<BITS, GS, 2, true>(a, st, zdim);
  return a.M <= 8 ? launch_gemv<BITS, GS, 1, false>(a, st, zdim) : launch_gemv<BITS, GS, 2, false>(a, st, zdim);
}

template <int BITS>
int dispatch_gs(const GemvArgs& a, int kgs, cudaStream_t st, int zdim) {
  switch (kgs) {
    case 32: return dispatch_mt<BITS, 32>(a, st, zdim);
    case 64: return dispatch_mt<BITS, 64>(a, st, zdim);
    default: return dispatch_mt<BITS, 128>(a, st, zdim);
  }
}

inline int pow2_floor(int v) {
  int p = 1;
  while (p * 2 <= v) p *= 2;
  return p;
}

}  // namespace

bool gptq_gemv_tma(const void* x, int x_dtype, long ldx, const int32_t* x_perm, const int32_t* qweight,
                   const int32_t* qzeros, const void* scales, int sc_dtype, const float* bias, void* out,
                   int out_dtype, long ldo, int M, int K, int N, int gs, int bits, float zoff, cudaStream_t st,
                   int* rc, void* workspace, size_t ws_bytes, const GemvFused* fu = nullptr);

// The TMA-fed GEMV when it takes the shape; else the register-fed kernel below, with the K split
// (cluster size) picked so the grid holds ~16 warps per SM.
int gptq_gemv(const void* x, int x_dtype, long ldx, const int32_t* x_perm, const int32_t* qweight,
              const int32_t* qzeros, const void* scales, int sc_dtype, const float* bias, void* out,
              int out_dtype, long ldo, int M, int K, int N, int gs, int bits, float zoff, cudaStream_t st,
              void* workspace, size_t ws_bytes) {
  int trc = 0;
  if (gptq_gemv_tma(x, x_dtype, ldx, x_perm, qweight, qzeros, scales, sc_dtype, bias, out, out_dtype, ldo, M, K, N,
                    gs, bits, zoff, st, &trc, workspace, ws_bytes))
    return trc;
  // kernel group: the largest of {128, 64, 32} dividing the checkpoint's group size
  const int kgs = (gs % 128 == 0) ? 128 : (gs % 64 == 0) ? 64 : 32;
  GemvArgs a = {};
  a.x = x; a.x_perm = x_perm; a.ldx = ldx; a.x_dtype = x_dtype;
  const int vec_elems = x_dtype == QL_F32 ? 4 : 8;
  a.x_vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (ldx % vec_elems == 0);
  a.qw = reinterpret_cast<const uint32_t*>(qweight);
  a.qz = reinterpret_cast<const uint32_t*>(qzeros);
  a.sc = scales; a.sc_dtype = sc_dtype; a.bias = bias;
  a.out = out; a.ldo = ldo; a.out_dtype = out_dtype;
  a.M = M; a.K = K; a.N = N;
  a.G = K / kgs;
  a.gs_mult = gs / kgs;
  a.lg_gs_mult = (a.gs_mult & (a.gs_mult - 1)) == 0 ? 31 - __builtin_clz(a.gs_mult) : -1;
  a.zoff = zoff;
  static int sms = 0, cs_cap = 0, warps_per_sm = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
    cs_cap = env_int("QL_GEMV_MAX_CLUSTER", 16);
    warps_per_sm = env_int("QL_GEMV_WARPS_PER_SM", 16);
  }
  const int cta_cols = (N + kCtaCols - 1) / kCtaCols;
  const int target = sms * (warps_per_sm / kNW);
  int cs = pow2_floor(target / cta_cols > 0 ? target / cta_cols : 1);
  if (cs > cs_cap) cs = cs_cap;
  if (cs > 16) cs = 16;
  while (cs > 1 && cs > a.G) cs /= 2;
  // keep the staged activation slice within shared memory
  while (cs < 16 && cs < a.G && (size_t)M * ((a.G + cs - 1) / cs) * kgs * 2 > 96 * 1024) cs *= 2;
  a.cs = cs;
  a.lg_cs = 31 - __builtin_clz(cs);
  return bits == 4 ? dispatch_gs<4>(a, kgs, st, 1) : dispatch_gs<8>(a, kgs, st, 1);
}

// Grouped (MoE) decode GEMV: one launch over every active expert. rows_per_expert_max bounds the
// rows any single expert holds (chooses 8- or 16-row chunks); max_active bounds the z extent.
int gptq_gemv_grouped(const void* x, int x_dtype, long ldx, const int32_t* x_rows, const int32_t* qweight,
                      const int32_t* qzeros, const void* scales, int sc_dtype, long qw_estride, long qz_estride,
                      long sc_estride, const int32_t* offsets, const int32_t* active, const int32_t* n_active,
                      int max_active, int rows_hint, void* out, int out_dtype, long ldo, int K, int N, int gs,
                      int bits, float zoff, cudaStream_t st, int glu) {
  const int kgs = (gs % 128 == 0) ? 128 : (gs % 64 == 0) ? 64 : 32;
  GemvArgs a = {};
  a.x = x; a.x_rows = x_rows; a.x_perm = nullptr; a.ldx = ldx; a.x_dtype = x_dtype;
  const int vec_elems = x_dtype == QL_F32 ? 4 : 8;
  a.x_vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (ldx % vec_elems == 0);
  a.qw = reinterpret_cast<const uint32_t*>(qweight);
  a.qz = reinterpret_cast<const uint32_t*>(qzeros);
  a.sc = scales; a.sc_dtype = sc_dtype; a.bias = nullptr;
  a.out = out; a.ldo = ldo; a.out_dtype = out_dtype;
  a.M = rows_hint <= 8 ? 8 : 16;   // chunk size: selects MT and sizes shared memory
  a.K = K; a.N = N;
  a.G = K / kgs;
  a.gs_mult = gs / kgs;
  a.lg_gs_mult = (a.gs_mult & (a.gs_mult - 1)) == 0 ? 31 - __builtin_clz(a.gs_mult) : -1;
  a.zoff = zoff;
  a.moe_offsets = offsets; a.moe_active = active; a.moe_n_active = n_active;
  a.glu = glu;
  a.qw_estride = qw_estride; a.qz_estride = qz_estride; a.sc_estride = sc_estride;
  int sms = 148, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int cta_cols = (N + kCtaCols - 1) / kCtaCols;
  const int target = sms * 4;
  const int per = cta_cols * (max_active > 0 ? max_active : 1);
  int cs = pow2_floor(target / per > 0 ? target / per : 1);
  if (cs > 8) cs = 8;
  while (cs > 1 && cs > a.G) cs /= 2;
  while (cs < 16 && cs < a.G && (size_t)a.M * ((a.G + cs - 1) / cs) * kgs * 2 > 96 * 1024) cs *= 2;
  a.cs = cs;
  a.lg_cs = 31 - __builtin_clz(cs);
  return bits == 4 ? dispatch_gs<4>(a, kgs, st, max_active) : dispatch_gs<8>(a, kgs, st, max_active);
}

}  // namespace ql

// =======================================================================================
// C ABI
// =======================================================================================
using namespace ql;

static int check_dtype(int d, const char* what) {
  if (d == QL_F32 || d == QL_F16 || d == QL_BF16) return QL_OK;
  set_error("%s: unknown dtype code %d", what, d);
  return QL_ERR_ARG;
}

static int check_gptq_dims(const char* fn, int K, int N, int gs, int bits) {
  if (bits != 4 && bits != 8) {
    set_error("%s: bits must be 4 or 8 (got %d)", fn, bits);
    return QL_ERR_UNSUPPORTED;
  }
  const int per = 32 / bits;
  if (K <= 0 || N <= 0 || gs <= 0) {
    set_error("%s: K, N and gs must be positive (K=%d N=%d gs=%d)", fn, K, N, gs);
    return QL_ERR_ARG;
  }
  if (K % gs != 0 || K % per != 0 || N % per != 0) {
    set_error("%s: dims must divide group/pack size (K=%d N=%d gs=%d bits=%d)", fn, K, N, gs, bits);
    return QL_ERR_ARG;
  }
  return QL_OK;
}

extern "C" int ql_gptq_dequant(const int32_t* qweight, const int32_t* qzeros, const void* scales,
                               int scales_dtype, const int32_t* g_idx, float* W, int K, int N, int gs,
                               int bits, float zero_offset, void* stream) {
  int rc = check_gptq_dims("ql_gptq_dequant", K, N, gs, bits);
  if (rc) return rc;
  if ((rc = check_dtype(scales_dtype, "ql_gptq_dequant(scales)"))) return rc;
  if (!qweight || !qzeros || !scales || !W) {
    set_error("ql_gptq_dequant: null pointer");
    return QL_ERR_ARG;
  }
  const long total = (long)(K / (32 / bits)) * N;
  const int threads = 256;
  const long blocks = (total + threads - 1) / threads;
  gptq_dequant_kernel<<<(unsigned)(blocks < 148 * 32 ? blocks : 148 * 32), threads, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint32_t*>(qweight), reinterpret_cast<const uint32_t*>(qzeros), scales,
      scales_dtype, g_idx, W, K, N, gs, bits, (double)zero_offset);
  return cuda_status(cudaGetLastError(), "ql_gptq_dequant launch");
}

extern "C" int ql_gptq_sort_rows(const int32_t* qweight_in, const int32_t* perm, int32_t* qweight_out,
                                 int K, int N, int bits, void* stream) {
  if (bits != 4 && bits != 8) {
    set_error("ql_gptq_sort_rows: bits must be 4 or 8 (got %d)", bits);
    return QL_ERR_UNSUPPORTED;
  }
  if (!qweight_in || !perm || !qweight_out || K <= 0 || N <= 0 || K % (32 / bits)) {
    set_error("ql_gptq_sort_rows: bad arguments (K=%d N=%d bits=%d)", K, N, bits);
    return QL_ERR_ARG;
  }
  if (qweight_in == qweight_out) {
    set_error("ql_gptq_sort_rows: input and output must not alias");
    return QL_ERR_ARG;
  }
  const long total = (long)(K / (32 / bits)) * N;
  const int threads = 256;
  const long blocks = (total + threads - 1) / threads;
  gptq_sort_rows_kernel<<<(unsigned)(blocks < 148 * 32 ? blocks : 148 * 32), threads, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint32_t*>(qweight_in), perm, reinterpret_cast<uint32_t*>(qweight_out), K, N, bits);
  return cuda_status(cudaGetLastError(), "ql_gptq_sort_rows launch");
}

namespace ql {
int gptq_gemm_sm100(const void* x, int x_dtype, long ldx, const int32_t* x_perm, const int32_t* qweight,
                    const int32_t* qzeros, const void* scales, int sc_dtype, const float* bias, void* out,
                    int out_dtype, long ldo, int M, int K, int N, int gs, int bits, float zoff, cudaStream_t st,
                    void* workspace, size_t ws_bytes, bool* handled);
}

namespace ql {
int gptq_matmul_impl(const void* x, int x_dtype, long ldx, const int32_t* x_perm, const int32_t* qweight,
                     const int32_t* qzeros, const void* scales, int scales_dtype, const float* bias, void* out,
                     int out_dtype, long ldo, int M, int K, int N, int gs, int bits, float zero_offset,
                     void* stream, void* workspace, size_t ws_bytes);
}

extern "C" int ql_gptq_matmul(const void* x, int x_dtype, long ldx, const int32_t* x_perm,
                              const int32_t* qweight, const int32_t* qzeros, const void* scales,
                              int scales_dtype, const float* bias, void* out, int out_dtype, long ldo,
                              int M, int K, int N, int gs, int bits, float zero_offset, void* stream) {
  return gptq_matmul_impl(x, x_dtype, ldx, x_perm, qweight, qzeros, scales, scales_dtype, bias, out, out_dtype,
                          ldo, M, K, N, gs, bits, zero_offset, stream, nullptr, 0);
}

extern "C" int ql_gptq_matmul_ws(const void* x, int x_dtype, long ldx, const int32_t* x_perm,
                                 const int32_t* qweight, const int32_t* qzeros, const void* scales,
                                 int scales_dtype, const float* bias, void* out, int out_dtype, long ldo,
                                 int M, int K, int N, int gs, int bits, float zero_offset, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  return gptq_matmul_impl(x, x_dtype, ldx, x_perm, qweight, qzeros, scales, scales_dtype, bias, out, out_dtype,
                          ldo, M, K, N, gs, bits, zero_offset, stream, workspace, workspace_bytes);
}

int ql::gptq_matmul_impl(const void* x, int x_dtype, long ldx, const int32_t* x_perm, const int32_t* qweight,
                         const int32_t* qzeros, const void* scales, int scales_dtype, const float* bias, void* out,
                         int out_dtype, long ldo, int M, int K, int N, int gs, int bits, float zero_offset,
                         void* stream, void* workspace, size_t ws_bytes) {
  int rc = check_gptq_dims("ql_gptq_matmul", K, N, gs, bits);
  if (rc) return rc;
  if ((rc = check_dtype(x_dtype, "ql_gptq_matmul(x)"))) return rc;
  if ((rc = check_dtype(scales_dtype, "ql_gptq_matmul(scales)"))) return rc;
  if ((rc = check_dtype(out_dtype, "ql_gptq_matmul(out)"))) return rc;
  if (M < 0) {
    set_error("ql_gptq_matmul: M must be >= 0 (got %d)", M);
    return QL_ERR_ARG;
  }
  if (M == 0) return QL_OK;
  if (!x || !qweight || !qzeros || !scales || !out) {
    set_error("ql_gptq_matmul: null pointer");
    return QL_ERR_ARG;
  }
  if (ldx < K || ldo < N) {
    set_error("ql_gptq_matmul: row strides too small (ldx=%ld K=%d ldo=%ld N=%d)", ldx, K, ldo, N);
    return QL_ERR_ARG;
  }
  if (gs % 32 != 0) {
    set_error("ql_gptq_matmul: group size %d is not a multiple of 32", gs);
    return QL_ERR_UNSUPPORTED;
  }
  if (N % 8 != 0) {
    set_error("ql_gptq_matmul: N=%d must be a multiple of 8", N);
    return QL_ERR_UNSUPPORTED;
  }
  if (!(zero_offset == 0.f || zero_offset == 1.f)) {
    set_error("ql_gptq_matmul: zero_offset must be 0 or 1 (got %g)", (double)zero_offset);
    return QL_ERR_UNSUPPORTED;
  }
  if ((reinterpret_cast<uintptr_t>(qweight) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(scales) & 15) != 0) {
    set_error("ql_gptq_matmul: qweight and scales must be 16-byte aligned");
    return QL_ERR_ALIGN;
  }
  cudaStream_t st = (cudaStream_t)stream;
  bool handled = false;
  rc = gptq_gemm_sm100(x, x_dtype, ldx, x_perm, qweight, qzeros, scales, scales_dtype, bias, out, out_dtype,
                       ldo, M, K, N, gs, bits, zero_offset, st, workspace, ws_bytes, &handled);
  if (handled || rc) return rc;
  // decode path: chunks of up to 16 tokens per launch
  for (int m0 = 0; m0 < M; m0 += 16) {
    const int mc = (M - m0) < 16 ? (M - m0) : 16;
    const char* xb = reinterpret_cast<const char*>(x) + (long)m0 * ldx * (x_dtype == QL_F32 ? 4 : 2);
    char* ob = reinterpret_cast<char*>(out) + (long)m0 * ldo * (out_dtype == QL_F32 ? 4 : 2);
    rc = gptq_gemv(xb, x_dtype, ldx, x_perm, qweight, qzeros, scales, scales_dtype, bias, ob, out_dtype, ldo,
                   mc, K, N, gs, bits, zero_offset, st, workspace, ws_bytes);
    if (rc) return rc;
  }
  return QL_OK;
}
