// GPTQ decode GEMV, TMA-fed: the packed weights stream through a shared-memory ring filled by
// a producer warp with tensor-memory-accelerator (TMA) copies, so every CTA keeps its whole
// ring (64-128 KB) in flight regardless of how long the consumer warps take per tile.
//
// Same arithmetic as the register-fed GEMV (gptq_gemv.cu): nibbles -> exact fp16 (q - z - off)
// with one LOP3 + one HSUB2/HFMA2, dot products and the 4-lane K reduction on mma.sync with
// register operands, per-group fp32 scaling, split-K over a thread-block cluster reduced in
// distributed shared memory.
//
// Layout of one ring stage (128 values of K for the CTA's 256 columns): a 3-D TMA box over the
// packed weight viewed as [N/32 strips][K/per rows][32 columns], i.e. per 32-column strip a
// [rows][128 B] block stored with the 128-byte swizzle (16-byte chunk c of row r lands at
// chunk c ^ (r % 8)). Consumer warp w reads strip w; lane (g, t) of step s reads the 16 bytes
// of row 4s + t, chunk g, so a warp touches 4 rows x 128 B with at most 2-way bank conflicts.
#include <cooperative_groups.h>
#include <cuda.h>

#include "ql_common.cuh"
#include "sm100_ptx.cuh"

namespace cg = cooperative_groups;

namespace ql {

// set when a bounded wait of this file's kernels gave up (read by ql_device_status)
__device__ int g_tma_gemv_status = 0;

int take_tma_gemv_status() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_tma_gemv_status, sizeof(int));
  const int zero = 0;
  cudaMemcpyToSymbol(g_tma_gemv_status, &zero, sizeof(int));
  return v;
}

namespace {

constexpr int kCW = 8;                 // consumer warps (one 32-column strip each)
constexpr int kThreads = (kCW + 1) * 32;
constexpr int kTileCols = kCW * 32;    // 256 columns per CTA
constexpr int kStageK = 128;           // K per ring stage

struct TmaGemvArgs {
  const void* x;
  const int32_t* x_perm;
  long ldx;
  int x_dtype;
  int x_vec;
  const uint32_t* qz;
  const void* sc;
  int sc_dtype;
  const float* bias;
  void* out;
  long ldo;
  int out_dtype;
  int M, K, N, gs;
  int nstage;   // K / kStageK
  int cs;       // cluster size along K
  float zoff;
};

template <int PER>
__device__ __forceinline__ int chunk_pos(int j) {
  return (j / PER) * PER + (j % PER % (PER / 2)) * 2 + (j % PER) / (PER / 2);
}

__device__ __forceinline__ void load_x8(const TmaGemvArgs& a, int m, int k, float (&v)[8]) {
  const long base = (long)m * a.ldx;
  if (a.x_perm == nullptr && a.x_vec) {
    if (a.x_dtype == QL_F16) {
      const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(a.x) + base + k);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(u32_as_h2(w[i]));
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    } else if (a.x_dtype == QL_BF16) {
      const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.x) + base + k);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    } else {
      const float4 f0 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.x) + base + k);
      const float4 f1 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.x) + base + k + 4);
      v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
      v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int src = a.x_perm ? a.x_perm[k + j] : k + j;
      v[j] = load_as_float(a.x, a.x_dtype, base + src);
    }
  }
}

// x[:, kbase : kbase + klen] -> power-of-two-scaled fp16 in unpack order (consumer warps only,
// synchronised with named barrier 1 so the producer warp keeps streaming).
template <int PER>
__device__ void stage_x(const TmaGemvArgs& a, int kbase, int klen, __half* xs, int* sh_exp, unsigned* sh_max,
                        int ctid, int nthr) {
  const int M = a.M;
  const int cpr = klen / 8;
  for (int m = 0; m < M; ++m) {
    float mx = 0.f;
    for (int kc = ctid; kc < cpr; kc += nthr) {
      float v[8];
      load_x8(a, m, kbase + kc * 8, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(v[j]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((ctid & 31) == 0) atomicMax(&sh_max[m], __float_as_uint(mx));
  }
  asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
  if (ctid < M) sh_exp[ctid] = stage_exponent(__uint_as_float(sh_max[ctid]));
  asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
  for (int idx = ctid; idx < M * cpr; idx += nthr) {
    const int m = idx / cpr, kc = idx - m * cpr;
    float v[8];
    load_x8(a, m, kbase + kc * 8, v);
    const float s = exp2i(-sh_exp[m]);
    __align__(16) __half h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) h[chunk_pos<PER>(j)] = __float2half_rn(v[j] * s);
    *reinterpret_cast<uint4*>(xs + (long)m * klen + kc * 8) = *reinterpret_cast<uint4*>(h);
  }
  asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
}

__device__ __forceinline__ void unpack_int4(uint32_t w, uint32_t zlo, uint32_t zhi, uint32_t (&P)[4]) {
  const __half2 one16 = __floats2half2_rn(0.0625f, 0.0625f);
  const uint32_t w8 = w >> 8;
  const uint32_t v0 = lop3_andor(w, 0x000F000Fu, kMagicF16x2);
  const uint32_t v1 = lop3_andor(w, 0x00F000F0u, kMagicF16x2);
  const uint32_t v2 = lop3_andor(w8, 0x000F000Fu, kMagicF16x2);
  const uint32_t v3 = lop3_andor(w8, 0x00F000F0u, kMagicF16x2);
  P[0] = h2_as_u32(__hsub2(u32_as_h2(v0), u32_as_h2(zlo)));
  P[1] = h2_as_u32(__hfma2(u32_as_h2(v1), one16, u32_as_h2(zhi)));
  P[2] = h2_as_u32(__hsub2(u32_as_h2(v2), u32_as_h2(zlo)));
  P[3] = h2_as_u32(__hfma2(u32_as_h2(v3), one16, u32_as_h2(zhi)));
}
__device__ __forceinline__ void unpack_int8(uint32_t w, uint32_t zlo, uint32_t (&P)[2]) {
  const uint32_t v0 = lop3_andor(w, 0x00FF00FFu, kMagicF16x2);
  const uint32_t v1 = lop3_andor(w >> 8, 0x00FF00FFu, kMagicF16x2);
  P[0] = h2_as_u32(__hsub2(u32_as_h2(v0), u32_as_h2(zlo)));
  P[1] = h2_as_u32(__hsub2(u32_as_h2(v1), u32_as_h2(zlo)));
}

template <int BITS, int NST>
struct TmaLayout {
  static constexpr int PER = 32 / BITS;
  static constexpr int ROWS = kStageK / PER;               // packed rows per stage
  static constexpr int kStripBytes = ROWS * 128;
  static constexpr int kStageBytes = kCW * kStripBytes;    // 16 KB (int4) / 32 KB (int8)
  static constexpr int kBarOff = NST * kStageBytes;
  static constexpr int kXsOff = kBarOff + 2 * NST * 8 + 16;   // + abort flag
};

template <int BITS, int GS, int MT, int NST>
__global__ void __launch_bounds__(kThreads, 1)
    gptq_gemv_tma_kernel(const __grid_constant__ CUtensorMap tmap_w, const TmaGemvArgs a) {
  using L = TmaLayout<BITS, NST>;
  constexpr int PER = L::PER;
  constexpr int GPS = kStageK / GS;                        // kernel groups per stage
  constexpr int SPG = GS / (4 * PER);                      // 4-row steps per group
  constexpr int MAXM = 8 * MT;
  constexpr uint32_t MASK = (1u << BITS) - 1u;

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ int sh_exp[16];
  __shared__ unsigned sh_max[16];
  const uint32_t sbase = ptx::smem_addr(smem);
  const uint32_t bar_full = sbase + L::kBarOff;
  const uint32_t bar_empty = bar_full + 8 * NST;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kBarOff + 16 * NST);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int rank = blockIdx.x;
  const int s0 = (int)((long)a.nstage * rank / a.cs);
  const int s1 = (int)((long)a.nstage * (rank + 1) / a.cs);
  const int nst = s1 - s0;
  const int klen = nst * kStageK;
  const int klen_max = ((a.nstage + a.cs - 1) / a.cs) * kStageK;
  const int M = a.M, N = a.N;
  __half* xs = reinterpret_cast<__half*>(smem + L::kXsOff);
  float* red = reinterpret_cast<float*>(smem + L::kXsOff + ((M * klen_max * 2 + 15) & ~15));

  if (a.cs > 1) cluster_arrive_relaxed();
  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, kCW);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (tid < 16) sh_max[tid] = 0u;
  __syncthreads();

  if (warp == kCW) {
    // ------------------------------------------------------------ producer warp
    if (lane == 0) {
      ptx::tma_prefetch(&tmap_w);
      const int strip0 = blockIdx.y * kCW;
      int i = 0;
      bool ok = true;
      for (; i < nst; ++i) {
        const int s = i % NST;
        if (i == NST) pdl_trigger();
        if (!ptx::mbar_wait(bar_empty + 8 * s, ((i / NST) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        ptx::mbar_arrive_expect_tx(bar_full + 8 * s, L::kStageBytes);
        asm volatile(
            "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
            "[%2];" ::"r"(sbase + s * L::kStageBytes),
            "l"(reinterpret_cast<uint64_t>(&tmap_w)), "r"(bar_full + 8 * s), "r"(0), "r"((s0 + i) * L::ROWS),
            "r"(strip0)
            : "memory");
      }
      if (nst <= NST) pdl_trigger();
      if (!ok) {
        for (int j = i > NST ? i - NST : 0; j < i; ++j) ptx::mbar_wait_drain(bar_full + 8 * (j % NST), (j / NST) & 1);
      }
    }
  } else {
    // ------------------------------------------------------------ consumer warps
    const int gq = lane >> 2, t = lane & 3;
    const int c0 = blockIdx.y * kTileCols + warp * 32 + gq * 4;
    const bool col_ok = c0 < N;
    const int cc = col_ok ? c0 : 0;
    pdl_wait();   // x may be the previous kernel's output
    stage_x<PER>(a, s0 * kStageK, klen, xs, sh_exp, sh_max, tid, kCW * 32);

    float acc[2][MT][4];
#pragma unroll
    for (int p = 0; p < 2; ++p)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[p][mt][i] = 0.f;

    // scales / zeros of the next stage are fetched one stage ahead
    float scv[GPS][4];
    uint32_t zw[GPS];
    auto load_sz = [&](int stage_idx, float (&sv)[GPS][4], uint32_t (&zv)[GPS]) {
#pragma unroll
      for (int u = 0; u < GPS; ++u) {
        const int srow = ((s0 + stage_idx) * kStageK + u * GS) / a.gs;
        if (col_ok && stage_idx < nst) {
          if (a.sc_dtype == QL_F16) {
            const uint2 h = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(a.sc) + (long)srow * N + cc);
            const float2 f0 = __half22float2(u32_as_h2(h.x)), f1 = __half22float2(u32_as_h2(h.y));
            sv[u][0] = f0.x; sv[u][1] = f0.y; sv[u][2] = f1.x; sv[u][3] = f1.y;
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) sv[u][q] = load_as_float(a.sc, a.sc_dtype, (long)srow * N + cc + q);
          }
          zv[u] = a.qz[(long)srow * (N / PER) + cc / PER] >> (BITS * (cc % PER));
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) sv[u][q] = 0.f;
          zv[u] = 0;
        }
      }
    };
    load_sz(0, scv, zw);

    const uint32_t strip_base = sbase + warp * L::kStripBytes;
    for (int i = 0; i < nst; ++i) {
      const int s = i % NST;
      float nscv[GPS][4];
      uint32_t nzw[GPS];
      load_sz(i + 1, nscv, nzw);
      if (!ptx::mbar_wait(bar_full + 8 * s, (i / NST) & 1, abort_flag)) break;
      const uint32_t stage_base = strip_base + s * L::kStageBytes;
#pragma unroll
      for (int u = 0; u < GPS; ++u) {
        uint32_t zlo[4], zhi[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float z = (float)((zw[u] >> (BITS * q)) & MASK) + a.zoff;
          zlo[q] = h2_as_u32(__float2half2_rn(1024.f + z));
          zhi[q] = h2_as_u32(__float2half2_rn(-(64.f + z)));
        }
        float gacc[2][MT][4];
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int q = 0; q < 4; ++q) gacc[p][mt][q] = 0.f;
#pragma unroll
        for (int st = 0; st < SPG; ++st) {
          const int row = (u * SPG + st) * 4 + t;                  // packed row inside the stage
          const uint32_t addr = stage_base + row * 128 + ((gq ^ (row & 7)) << 4);
          uint4 wv;
          asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(wv.x), "=r"(wv.y), "=r"(wv.z), "=r"(wv.w)
                       : "r"(addr));
          const uint32_t wcol[4] = {wv.x, wv.y, wv.z, wv.w};
          const int koff = i * kStageK + row * PER;                // offset inside the staged x slice
          if constexpr (BITS == 4) {
            uint32_t P[4][4];
#pragma unroll
            for (int q = 0; q < 4; ++q) unpack_int4(wcol[q], zlo[q], zhi[q], P[q]);
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
            for (int q = 0; q < 4; ++q) unpack_int8(wcol[q], zlo[q], P[q]);
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
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            acc[p][mt][0] = fmaf(scv[u][2 * p], gacc[p][mt][0], acc[p][mt][0]);
            acc[p][mt][1] = fmaf(scv[u][2 * p], gacc[p][mt][1], acc[p][mt][1]);
            acc[p][mt][2] = fmaf(scv[u][2 * p + 1], gacc[p][mt][2], acc[p][mt][2]);
            acc[p][mt][3] = fmaf(scv[u][2 * p + 1], gacc[p][mt][3], acc[p][mt][3]);
          }
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_empty + 8 * s);
#pragma unroll
      for (int u = 0; u < GPS; ++u) {
        zw[u] = nzw[u];
#pragma unroll
        for (int q = 0; q < 4; ++q) scv[u][q] = nscv[u][q];
      }
    }

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
    } else {
      // partials pushed into the owning rank's shared memory (rank q owns columns
      // [q * cpo, (q + 1) * cpo) of the CTA tile, cpo = 256 / cs)
      cg::cluster_group cluster = cg::this_cluster();
      const int lg_cs = 31 - __clz(a.cs);
      const int lg_cpo = 8 - lg_cs;
      const int chunk = (kTileCols >> lg_cs) * MAXM;
      __syncwarp();
      cluster_wait_acquire();
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int lcol = warp * 32 + gq * 4 + 2 * p;
        const int owner = lcol >> lg_cpo;
        float* dst = cluster.map_shared_rank(red, owner) + rank * chunk + (lcol - (owner << lg_cpo)) * MAXM;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int tok = 8 * mt + 2 * t + (i & 1);
            if (tok < M) dst[(i >> 1) * MAXM + tok] = acc[p][mt][i] * exp2i(sh_exp[tok]);
          }
      }
    }
  }

  __syncwarp();  // cluster barriers are .aligned: every warp reaches them converged
  if (a.cs > 1) {
    if (warp == kCW) cluster_wait_acquire();   // the producer joins the cluster barrier phases
    cluster_arrive_release();
    cluster_wait_acquire();
    const int lg_cs = 31 - __clz(a.cs);
    const int cpo = kTileCols >> lg_cs;
    const int chunk = cpo * MAXM;
    for (int s = tid; s < cpo * M; s += blockDim.x) {
      const int c = s / M, tok = s - c * M;
      float v = 0.f;
      for (int q = 0; q < a.cs; ++q) v += red[q * chunk + c * MAXM + tok];
      const int col = blockIdx.y * kTileCols + rank * cpo + c;
      if (col < N) {
        if (a.bias) v += a.bias[col];
        store_from_float(a.out, a.out_dtype, (long)tok * a.ldo + col, v);
      }
    }
  }
  if (tid == 0 && *abort_flag) atomicExch(&g_tma_gemv_status, 1);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

template <int BITS, int GS, int MT, int NST>
int launch_tma(const TmaGemvArgs& a, const uint32_t* qweight, cudaStream_t st) {
  using L = TmaLayout<BITS, NST>;
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    set_error("ql_gptq_matmul: cuTensorMapEncodeTiled is unavailable");
    return QL_ERR_CUDA;
  }
  CUtensorMap tmap;
  const cuuint64_t dims[3] = {32, (cuuint64_t)(a.K / L::PER), (cuuint64_t)(a.N / 32)};
  const cuuint64_t strides[2] = {(cuuint64_t)a.N * 4, 128};
  const cuuint32_t box[3] = {32, (cuuint32_t)L::ROWS, (cuuint32_t)kCW};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint32_t*>(qweight), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return -1;  // not expressible as a tensor map: caller falls back
  auto kern = gptq_gemv_tma_kernel<BITS, GS, MT, NST>;
  const int klen_max = ((a.nstage + a.cs - 1) / a.cs) * kStageK;
  const size_t smem = 1024 + L::kXsOff + (((size_t)a.M * klen_max * 2 + 15) & ~(size_t)15) +
                      (size_t)kTileCols * 8 * MT * 4;
  if (smem > 200 * 1024) return -1;  // too large an activation slice: caller falls back
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024),
                         "cudaFuncSetAttribute(tma gemv smem)");
    if (rc) return rc;
    rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                     "cudaFuncSetAttribute(tma gemv cluster)");
    if (rc) return rc;
    configured_dev = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.cs, (a.N + kTileCols - 1) / kTileCols, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
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
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, tmap, a), "gptq_gemv_tma launch");
}

template <int BITS, int GS>
int tma_mt(const TmaGemvArgs& a, const uint32_t* qw, cudaStream_t st) {
  constexpr int NST = BITS == 4 ? 4 : 3;
  return a.M <= 8 ? launch_tma<BITS, GS, 1, NST>(a, qw, st) : launch_tma<BITS, GS, 2, NST>(a, qw, st);
}

template <int BITS>
int tma_gs(const TmaGemvArgs& a, int kgs, const uint32_t* qw, cudaStream_t st) {
  switch (kgs) {
    case 32: return tma_mt<BITS, 32>(a, qw, st);
    case 64: return tma_mt<BITS, 64>(a, qw, st);
    default: return tma_mt<BITS, 128>(a, qw, st);
  }
}

inline int pow2_floor(int v) {
  int p = 1;
  while (p * 2 <= v) p *= 2;
  return p;
}

}  // namespace

// Returns true (and the launch status in *rc) when the TMA-fed GEMV handles this shape.
bool gptq_gemv_tma(const void* x, int x_dtype, long ldx, const int32_t* x_perm, const int32_t* qweight,
                   const int32_t* qzeros, const void* scales, int sc_dtype, const float* bias, void* out,
                   int out_dtype, long ldo, int M, int K, int N, int gs, int bits, float zoff, cudaStream_t st,
                   int* rc) {
  static int enabled = -1, sms = 0, ctas_per_sm = 0;
  if (enabled < 0) {
    enabled = env_int("QL_GEMV_TMA", 0);
    ctas_per_sm = env_int("QL_GEMV_TMA_CTAS_PER_SM", 2);
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  if (!enabled || N % 32 != 0 || K % kStageK != 0 || (gs % 128 != 0 && gs != 32 && gs != 64)) return false;
  if ((reinterpret_cast<uintptr_t>(qweight) & 15) != 0) return false;
  const int kgs = gs % 128 == 0 ? 128 : gs;
  TmaGemvArgs a;
  a.x = x; a.x_perm = x_perm; a.ldx = ldx; a.x_dtype = x_dtype;
  const int vec_elems = x_dtype == QL_F32 ? 4 : 8;
  a.x_vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (ldx % vec_elems == 0);
  a.qz = reinterpret_cast<const uint32_t*>(qzeros);
  a.sc = scales; a.sc_dtype = sc_dtype; a.bias = bias;
  a.out = out; a.ldo = ldo; a.out_dtype = out_dtype;
  a.M = M; a.K = K; a.N = N; a.gs = gs; a.zoff = zoff;
  a.nstage = K / kStageK;
  const int tiles = (N + kTileCols - 1) / kTileCols;
  int cs = pow2_floor(sms * ctas_per_sm / tiles > 0 ? sms * ctas_per_sm / tiles : 1);
  if (cs > 16) cs = 16;
  while (cs > 1 && cs > a.nstage) cs /= 2;
  while (cs < 16 && cs < a.nstage && (size_t)M * ((a.nstage + cs - 1) / cs) * kStageK * 2 > 64 * 1024) cs *= 2;
  a.cs = cs;
  const int r = bits == 4 ? tma_gs<4>(a, kgs, reinterpret_cast<const uint32_t*>(qweight), st)
                          : tma_gs<8>(a, kgs, reinterpret_cast<const uint32_t*>(qweight), st);
  if (r < 0) return false;
  *rc = r;
  return true;
}

}  // namespace ql
