// GGUF Q4_K decode GEMV / small-M GEMM, TMA-fed, on the integer tensor-core MMA.
//
// Reference semantics (webtorch/ggufload.py:120-131, 190-202; GGMLLinear.forward
// webtorch/_core.py:4399-4406): row n of the [N, K] weight is K/256 super-blocks of 144 bytes,
// f16 d | f16 dmin | scales[12] | qs[128]; sub-block j (32 values) has a 6-bit scale sc_j and
// min m_j, value = d*sc_j * q - dmin*m_j, q the low nibbles of qs[32G .. 32G+31] for j = 2G and
// the high nibbles for j = 2G+1.
//
// Layout in flight: the raw buffer is read in place as a [N rows][K/256 * 144 bytes] byte
// tensor. A ring stage is one super-block of the CTA's 128 rows (a 2-D TMA box of 144 bytes x
// 128 rows, 18 KB, rows 144 bytes apart in shared memory: the 8 x 4 lanes of a warp then hit 32
// distinct banks). One producer warp issues the copies; 8 consumer warps own 16 rows each.
//
// Arithmetic: mma.sync m16n8k32 with u8 weights x s8 activation bytes. The low (high) nibbles
// of a lane's words at bytes 4t and 16 + 4t of quant group G are the A fragment of sub-block
// 2G (2G + 1) with one mask each. Activations are staged as 23-bit integers with one
// power-of-two exponent per token and super-block (gemv_common.cuh, stage_x3), three signed byte
// planes in three MMA columns per token, with exact per-sub-block sums S of the staged integers.
// Per row, token and plane pair ((b2, b1) or (0, b0)), sub-block j adds
//   P += sc_j * (256 C_hi + C_lo)   (as exact int32 sums of sc_j C_hi and sc_j C_lo)
//   Q += m_j * S_j                  (int32, exact)
// and each super-block ends with acc += 2^e (d * P - dmin * Q); the two plane-pair lanes are
// added (the first times 2^8) at the end. The 16 six-bit scales and mins of a row are unpacked
// four at a time with byte-parallel masks (get_scale_min_k4 on whole words).
//
// Split-K runs over a thread-block cluster; partial sums go to the owning rank's shared memory
// with st.async stores that count down its mbarrier. More than 4 tokens: activations staged once
// in global memory, chunks of 8 tokens as independent z-slices of the grid (the first slice
// reads the weights from HBM, the rest mostly from L2).
#include <cuda.h>

#include "gemv_common.cuh"
#include "sm100_ptx.cuh"

namespace ql {

// set when a bounded wait of this file's kernel gave up (read by ql_device_status)
__device__ int g_q4k_tma_status = 0;

int take_q4k_tma_status() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_q4k_tma_status, sizeof(int));
  const int zero = 0;
  cudaMemcpyToSymbol(g_q4k_tma_status, &zero, sizeof(int));
  return v;
}

namespace {

constexpr int kCW = 8;                    // consumer warps
constexpr int kThreads = (kCW + 1) * 32;
constexpr int kRows = 16 * kCW;           // rows per CTA (one 16-row MMA tile per warp)
constexpr int kBlkVals = 256;
constexpr int kBlkBytes = 144;
constexpr int kStageBytes = kRows * kBlkBytes;   // 18432: one super-block of every row

struct Q4kTmaArgs {
  const void* x;
  long ldx;
  int x_dtype;
  int x_vec;
  const float* bias;
  void* out;
  long ldo;
  int out_dtype;
  int M, K, N;
  int nb;       // super-blocks per row
  int cs;       // cluster size along K
  int mchunk;   // tokens per z-slice
  int nst;      // ring stages (the kernel's NST)
  // activations staged in global memory (more than 4 tokens): chunk of z-slice c at
  // xg + c * chunk_bytes (B operand of all K, then the per-super-block sums at sum_off)
  const uint8_t* xg;
  long chunk_bytes, sum_off;
  // up to 4 tokens with 16-byte aligned rows of x: the producer copies the CTA's slice of x into
  // shared memory by bulk copy ahead of the weights (xsize = bytes per element; pdl = launched
  // as a programmatic dependent, so x is copied after the first ring fill)
  int xbulk, xsize, pdl;
};

// activation source in the form gemv::load_x8 reads
struct XSrc {
  const void* x;
  const int32_t* x_rows;
  const int32_t* x_perm;
  long ldx;
  int x_dtype;
  int x_vec;
  int M;
  int glu;
  const float* nw;   // RMSNorm weight folded into the loads (unused here: NULL)
  const float* nr;
  float norm_eps;
};

// Ring stage: the weights' TMA box, then with XP (activations staged in global memory) the
// stage's B operand (8 steps x 4 lanes x kXSlots slots x 8 bytes) and its sums record.
template <int NST, int MAXM, bool XP>
struct Layout {
  static constexpr int kXSlots = gemv::xb3_slots(MAXM);
  static constexpr int kXBytes = XP ? kBlkVals * kXSlots : 0;
  static constexpr int kSBytes = XP ? q4k_sum_ints(MAXM) * 4 : 0;
  static constexpr int kStage = kStageBytes + kXBytes + kSBytes;   // a multiple of 128
  static constexpr int kBarOff = NST * kStage;
  static constexpr int kXsOff = kBarOff + 2 * NST * 8 + 32;   // + reduction barrier, abort flag, x barrier
};

__device__ __forceinline__ void st_async_f32(uint32_t raddr, float v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr),
               "r"(__float_as_uint(v)), "r"(rbar)
               : "memory");
}

// NP MMA tiles of two tokens each. Two CTAs per SM: registers are allocated per pair of warps,
// so the 9 warps count as 10 and the limit is 96 registers per thread.
template <int NP, int NST, bool XP>
__global__ void __launch_bounds__(kThreads, 2)
    q4k_gemv_tma_kernel(const __grid_constant__ CUtensorMap tmap, const Q4kTmaArgs a) {
  constexpr int MAXM = 2 * NP;
  using L = Layout<NST, MAXM, XP>;
  static_assert(L::kStage % 128 == 0, "stage alignment");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = ptx::smem_addr(smem);
  const uint32_t bar_full = sbase + L::kBarOff;
  const uint32_t bar_empty = bar_full + 8 * NST;
  const uint32_t bar_red = bar_full + 16 * NST;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kBarOff + 16 * NST + 8);
  const uint32_t bar_x = bar_full + 16 * NST + 16;   // the bulk copy of x (xbulk)

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = blockIdx.x, cs = a.cs;
  const int tok0 = blockIdx.z * a.mchunk;
  const int M = min(a.mchunk, a.M - tok0);
  // this rank's super-blocks [b0, b0 + nbl)
  const int bq = a.nb / cs, brem = a.nb - bq * cs;
  const int b0 = rank * bq + min(rank, brem);
  const int nbl = bq + (rank < brem ? 1 : 0);
  const int nbl_max = bq + (brem ? 1 : 0);
  // staged activations (without XP): B rows of sstride slots; sub-block sums [2 M rows][gstride]
  // (row 2m: S of v1, 2m + 1: S of b0); factors [M][nbl_max] (fe bits per super-block)
  const int sstride = XP ? L::kXSlots : gemv::xb3_slots(M);
  const int gstride = nbl_max * 8 + 2;
  uint2* xb = reinterpret_cast<uint2*>(smem + L::kXsOff);
  const int xs_bytes = XP ? 0 : (nbl_max * kBlkVals * sstride + 15) & ~15;
  int* gsum = reinterpret_cast<int*>(smem + L::kXsOff + xs_bytes);
  const int gs_bytes = XP ? 0 : (2 * M * gstride * 4 + 15) & ~15;
  int* gexp = gsum + gs_bytes / 4;
  const int ge_bytes = XP ? 0 : (M * nbl_max * 4 + 15) & ~15;
  // xbulk: the raw rows of x for this CTA's super-blocks, nbl_max * 256 elements apart
  unsigned char* xraw = smem + L::kXsOff + xs_bytes + gs_bytes + ge_bytes;
  const int xr_bytes = a.xbulk ? (M * nbl_max * kBlkVals * a.xsize + 15) & ~15 : 0;
  // split-K partials received by this rank: [cs ranks][MAXM tokens][rows_max rows]; rank q
  // owns the CTA rows [orow(q), orow(q + 1)), orow(q) = ceil(q * kRows / cs)
  float* red = reinterpret_cast<float*>(smem + L::kXsOff + xs_bytes + gs_bytes + ge_bytes + xr_bytes);
  const int rows_max = (kRows + cs - 1) / cs;
  const int or0 = (rank * kRows + cs - 1) / cs, or1 = ((rank + 1) * kRows + cs - 1) / cs;

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, kCW);
    }
    ptx::mbar_init(bar_red, 1);
    ptx::mbar_init(bar_x, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    if (cs > 1) ptx::mbar_arrive_expect_tx(bar_red, (uint32_t)(cs * M * (or1 - or0) * 4));
  }
  __syncthreads();
  if (cs > 1) cluster_arrive_relaxed();   // waited for before the first remote store

  // the bulk copy of this CTA's x slice (one copy per token row)
  auto copy_x = [&]() {
    pdl_wait();   // x may be the previous kernel's output
    const uint32_t row_bytes = (uint32_t)(nbl * kBlkVals * a.xsize);
    ptx::mbar_arrive_expect_tx(bar_x, (uint32_t)M * row_bytes);
    const char* xs = reinterpret_cast<const char*>(a.x) + (size_t)b0 * kBlkVals * a.xsize;
    for (int m = 0; m < M; ++m)
      ptx::bulk_load(ptx::smem_addr(xraw + (size_t)m * nbl_max * kBlkVals * a.xsize),
                     xs + (size_t)(tok0 + m) * a.ldx * a.xsize, row_bytes, bar_x);
  };

  if (warp == kCW) {
    // ------------------------------------------------------------ producer warp
    if (lane == 0) {
      ptx::tma_prefetch(&tmap);
      const int row0 = blockIdx.y * kRows;
      const uint8_t* xgc = XP ? a.xg + (long)blockIdx.z * a.chunk_bytes : nullptr;
      if (XP) pdl_wait();   // the staged activations are the previous kernel's output
      // x goes first into the memory queue, unless this grid may start before the previous
      // kernel ends: then the weights (independent of it) go first and x after the ring's fill
      const bool x_first = a.xbulk && !a.pdl;
      const int x_after = a.xbulk && a.pdl ? min(NST, nbl) - 1 : -1;
      if (x_first) copy_x();
      int i = 0;
      bool ok = true;
      for (; i < nbl; ++i) {
        const int s = i % NST;
        if (i == NST) pdl_trigger();
        if (!ptx::mbar_wait(bar_empty + 8 * s, ((i / NST) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t fb = bar_full + 8 * s;
        const uint32_t st = sbase + s * L::kStage;
        ptx::mbar_arrive_expect_tx(fb, L::kStage);
        ptx::tma_load_2d(st, &tmap, fb, (b0 + i) * kBlkBytes, row0);
        if constexpr (XP) {
          ptx::bulk_load(st + kStageBytes, xgc + (long)(b0 + i) * L::kXBytes, L::kXBytes, fb);
          ptx::bulk_load(st + kStageBytes + L::kXBytes, xgc + a.sum_off + (long)(b0 + i) * L::kSBytes, L::kSBytes, fb);
        }
        if (i == x_after) copy_x();
      }
      if (nbl <= NST) pdl_trigger();
      if (!ok) {
        for (int j = i > NST ? i - NST : 0; j < i; ++j) ptx::mbar_wait_drain(bar_full + 8 * (j % NST), (j / NST) & 1);
        if (x_first || (x_after >= 0 && i > x_after)) ptx::mbar_wait_drain(bar_x, 0);
      }
    }
    __syncwarp();
    if (cs > 1) cluster_wait_acquire();   // pairs with the arrive above (every thread once)
  } else {
    // ------------------------------------------------------------ consumer warps
    // Lane (g, t): MMA rows g / g + 8 are CTA rows 16 w + g / 16 w + g + 8. In MMA tile mq, B
    // columns 4u .. 4u + 3 hold b2, b1, 0, b0 of token 2 mq + u; the lane's D columns 2t, 2t + 1
    // are the plane pair t % 2 ((b2, b1) or (0, b0)) of token 2 mq + t / 2.
    const int g = lane >> 2, t = lane & 3;
    const int ptok = t >> 1, pp = t & 1;
    const int btok = g >> 2, bpl = (g & 3) == 3 ? 2 : (g & 3);
    const bool bld = (g & 3) != 2;
    pdl_wait();   // x may be the previous kernel's output
    bool x_ok = true;
    if constexpr (!XP) {
      // int8 staging order = natural K order: a 32-K step's B fragment (t) holds K 4t .. 4t + 3
      // and 16 + 4t .. 16 + 4t + 3; sums per 32 values (one sub-block), exponents per super-block
      auto sums = [&](int m, int sb, int s1, int s0v) {
        gsum[(2 * m) * gstride + sb] = s1;
        gsum[(2 * m + 1) * gstride + sb] = s0v;
      };
      auto expo = [&](int m, int b, float fe) { gexp[m * nbl_max + b] = __float_as_int(fe); };
      if (a.xbulk) {
        // the slice of x arrives in shared memory by bulk copy; stage it from there
        x_ok = ptx::mbar_wait(bar_x, 0, abort_flag);
        const XSrc xsrc{xraw, nullptr, nullptr, (long)nbl_max * kBlkVals, a.x_dtype, 1, M, 0};
        gemv::stage_x3<8, 32, 256, true>(xsrc, 0, x_ok ? nbl * kBlkVals : 0, sstride, xb, sums, expo, tid, kCW * 32);
      } else {
        const XSrc xsrc{reinterpret_cast<const char*>(a.x) + (size_t)tok0 * a.ldx * (a.x_dtype == QL_F32 ? 4u : 2u),
                        nullptr, nullptr, a.ldx, a.x_dtype, a.x_vec, M, 0};
        gemv::stage_x3<8, 32, 256, true>(xsrc, b0 * kBlkVals, nbl * kBlkVals, sstride, xb, sums, expo, tid, kCW * 32);
      }
    }

    float acc[NP][2];
#pragma unroll
    for (int mq = 0; mq < NP; ++mq) acc[mq][0] = acc[mq][1] = 0.f;
    const int r0 = warp * 16 + g;
    const uint32_t xb_base = ptx::smem_addr(xb);
    for (int i = 0; i < (x_ok ? nbl : 0); ++i) {
      const int s = i % NST;
      if (!ptx::mbar_wait(bar_full + 8 * s, (i / NST) & 1, abort_flag)) break;
      const unsigned char* p0 = smem + s * L::kStage + r0 * kBlkBytes;
      // B operand and sums of this stage: staged in the ring (XP) or once for the CTA's slice
      const uint32_t xstage = XP ? sbase + s * L::kStage + kStageBytes : xb_base + i * 8 * 4 * sstride * 8;
      const int* sstage = XP ? reinterpret_cast<const int*>(smem + s * L::kStage + kStageBytes + L::kXBytes) : nullptr;
      const unsigned char* p1 = p0 + 8 * kBlkBytes;
      const uint4 h0 = *reinterpret_cast<const uint4*>(p0);
      const uint4 h1 = *reinterpret_cast<const uint4*>(p1);
      // six-bit scales / mins of sub-blocks 0-3 and 4-7, one per byte
      const uint32_t sc0[2] = {h0.y & 0x3F3F3F3Fu, (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u)};
      const uint32_t mn0[2] = {h0.z & 0x3F3F3F3Fu, ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u)};
      const uint32_t sc1[2] = {h1.y & 0x3F3F3F3Fu, (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u)};
      const uint32_t mn1[2] = {h1.z & 0x3F3F3F3Fu, ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u)};
      // exact int32 sums over the super-block, per token tile and row (0 / 1 = r0 / r0 + 8):
      //   PH / PL = 16 * sum_j sc_j * C_hi / C_lo (|.| < 2^29), Q = sum_j m_j * S_j (|.| < 2^28);
      // odd sub-blocks enter the MMA as 16 q, even ones as q with their scale taken 16 times
      int PH[NP][2], PL[NP][2], Q[NP][2];
#pragma unroll
      for (int mq = 0; mq < NP; ++mq)
#pragma unroll
        for (int r = 0; r < 2; ++r) PH[mq][r] = PL[mq][r] = Q[mq][r] = 0;
#pragma unroll
      for (int G = 0; G < 4; ++G) {
        const uint32_t w00 = *reinterpret_cast<const uint32_t*>(p0 + 16 + 32 * G + 4 * t);
        const uint32_t w01 = *reinterpret_cast<const uint32_t*>(p0 + 32 + 32 * G + 4 * t);
        const uint32_t w10 = *reinterpret_cast<const uint32_t*>(p1 + 16 + 32 * G + 4 * t);
        const uint32_t w11 = *reinterpret_cast<const uint32_t*>(p1 + 32 + 32 * G + 4 * t);
        int2 S2[NP];   // sums of sub-blocks 2G, 2G + 1 for the lane's token and plane pair
#pragma unroll
        for (int mq = 0; mq < NP; ++mq) {
          const int tok = 2 * mq + ptok;
          if constexpr (XP)
            S2[mq] = tok < M ? make_int2(sstage[(4 * G + pp) * MAXM + tok], sstage[(4 * G + 2 + pp) * MAXM + tok])
                             : make_int2(0, 0);
          else
            S2[mq] = tok < M ? *reinterpret_cast<const int2*>(gsum + (2 * tok + pp) * gstride + i * 8 + 2 * G)
                             : make_int2(0, 0);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int j = 2 * G + u;   // sub-block
          // low nibbles as q, high nibbles in place as 16 q (fits u8; rescaled at the end)
          const uint32_t msk = u ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
          const uint32_t a0 = w00 & msk, a1 = w10 & msk, a2 = w01 & msk, a3 = w11 & msk;
          const int s0 = (int)__byte_perm(sc0[j >> 2], 0u, 0x4440u + (j & 3)) << (u ? 0 : 4);
          const int s1 = (int)__byte_perm(sc1[j >> 2], 0u, 0x4440u + (j & 3)) << (u ? 0 : 4);
          const int m0 = (int)__byte_perm(mn0[j >> 2], 0u, 0x4440u + (j & 3));
          const int m1 = (int)__byte_perm(mn1[j >> 2], 0u, 0x4440u + (j & 3));
#pragma unroll
          for (int mq = 0; mq < NP; ++mq) {
            const int btk = 2 * mq + btok;
            uint32_t b0 = 0u, b1 = 0u;
            if (bld && btk < M) {
              const uint32_t xa = xstage + ((j * 4 + t) * sstride + 3 * btk + bpl) * 8;
              asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(xa));
            }
            int d[4] = {0, 0, 0, 0};
            mma_16832_u8s8(d, a0, a1, a2, a3, b0, b1);
            PH[mq][0] += s0 * d[0];
            PL[mq][0] += s0 * d[1];
            PH[mq][1] += s1 * d[2];
            PL[mq][1] += s1 * d[3];
            const int S = u ? S2[mq].y : S2[mq].x;
            Q[mq][0] += m0 * S;
            Q[mq][1] += m1 * S;
          }
        }
      }
      const float2 dd0 = __half22float2(u32_as_h2(h0.x));   // (d, dmin) of row r0
      const float2 dd1 = __half22float2(u32_as_h2(h1.x));   // and of row r0 + 8
#pragma unroll
      for (int mq = 0; mq < NP; ++mq) {
        const int tok = 2 * mq + ptok;
        float fe = 0.f;
        if (tok < M) fe = __int_as_float(XP ? sstage[16 * MAXM + tok] : gexp[tok * nbl_max + i]);
        const float P0 = 0.0625f * fmaf(256.f, (float)PH[mq][0], (float)PL[mq][0]);
        const float P1 = 0.0625f * fmaf(256.f, (float)PH[mq][1], (float)PL[mq][1]);
        acc[mq][0] = fmaf(dd0.x * fe, P0, fmaf(-dd0.y * fe, (float)Q[mq][0], acc[mq][0]));
        acc[mq][1] = fmaf(dd1.x * fe, P1, fmaf(-dd1.y * fe, (float)Q[mq][1], acc[mq][1]));
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_empty + 8 * s);
    }

    // the (b2, b1) lane's sums count 2^8 times the (0, b0) lane's; add the pair (exact scaling)
#pragma unroll
    for (int mq = 0; mq < NP; ++mq)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float v = pp ? acc[mq][h] : 256.f * acc[mq][h];
        acc[mq][h] = v + __shfl_xor_sync(0xffffffffu, v, 1);
      }
    if (cs == 1) {
#pragma unroll
      for (int mq = 0; mq < NP; ++mq) {
        const int tok = 2 * mq + ptok;
        if (pp == 0 && tok < M) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int row = blockIdx.y * kRows + r0 + 8 * h;
            if (row < a.N) {
              float v = acc[mq][h];
              if (a.bias) v += a.bias[row];
              store_from_float(a.out, a.out_dtype, (long)(tok0 + tok) * a.ldo + row, v);
            }
          }
        }
      }
    } else {
      __syncwarp();
      cluster_wait_acquire();   // every CTA of the cluster has initialised its mbarriers
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = r0 + 8 * h;
        const int owner = (r * cs) / kRows;
        const int orow = (owner * kRows + cs - 1) / cs;
        const uint32_t rb = ptx::mapa(ptx::smem_addr(red), owner);
        const uint32_t rbar = ptx::mapa(bar_red, owner);
#pragma unroll
        for (int mq = 0; mq < NP; ++mq) {
          const int tok = 2 * mq + ptok;
          if (pp == 0 && tok < M) st_async_f32(rb + ((rank * MAXM + tok) * rows_max + (r - orow)) * 4, acc[mq][h], rbar);
        }
      }
    }
  }

  if (cs > 1) {
    // reduce the owned rows over the ranks in rank order (deterministic) and store
    const bool got = ptx::mbar_wait(bar_red, 0, abort_flag);
    const int nrow = or1 - or0;
    if (got) {
      for (int s = tid; s < nrow * M; s += blockDim.x) {
        const int tok = s / nrow, r = s - tok * nrow;
        float v = 0.f;
        for (int q = 0; q < cs; ++q) v += red[(q * MAXM + tok) * rows_max + r];
        const int row = blockIdx.y * kRows + or0 + r;
        if (row < a.N) {
          if (a.bias) v += a.bias[row];
          store_from_float(a.out, a.out_dtype, (long)(tok0 + tok) * a.ldo + row, v);
        }
      }
    }
  }
  if (tid == 0 && *abort_flag) atomicExch(&g_q4k_tma_status, 1);
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

constexpr int kNST = 4;
constexpr int kXpTokens = 8;   // tokens per z-slice when the activations are staged in global memory

// dynamic shared memory of one CTA with an nst-stage ring for z-slices of mchunk tokens, as the
// kernel carves it up (xp: activations staged in global memory and carried by the ring)
size_t smem_bytes(int mchunk, int nb, int cs, int nst, bool xp, int xbulk_size = 0) {
  const int nbl_max = (nb + cs - 1) / cs;
  const int maxm = xp ? kXpTokens : (mchunk <= 2 ? 2 : 4);
  const size_t red = cs > 1 ? (size_t)cs * maxm * ((kRows + cs - 1) / cs) * 4 : 0;
  if (xp) {
    const size_t stage = kStageBytes + (size_t)kBlkVals * gemv::xb3_slots(kXpTokens) + q4k_sum_ints(kXpTokens) * 4;
    return 1024 + (size_t)nst * stage + 2 * nst * 8 + 32 + red;
  }
  const size_t xs = ((size_t)nbl_max * kBlkVals * gemv::xb3_slots(mchunk) + 15) & ~(size_t)15;
  const size_t gsb = ((size_t)2 * mchunk * (nbl_max * 8 + 2) * 4 + 15) & ~(size_t)15;
  const size_t geb = ((size_t)mchunk * nbl_max * 4 + 15) & ~(size_t)15;
  const size_t xrb = ((size_t)mchunk * nbl_max * kBlkVals * xbulk_size + 15) & ~(size_t)15;
  return 1024 + (size_t)nst * kStageBytes + 2 * nst * 8 + 32 + xs + gsb + geb + xrb + red;
}

template <int NP, int NST, bool XP>
int launch(const Q4kTmaArgs& a, const uint8_t* raw, size_t smem, cudaStream_t st) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return -1;
  CUtensorMap tm;
  const cuuint64_t rowbytes = (cuuint64_t)a.nb * kBlkBytes;
  const cuuint64_t dims[2] = {rowbytes, (cuuint64_t)a.N};
  const cuuint64_t strides[1] = {rowbytes};
  const cuuint32_t box[2] = {kBlkBytes, kRows};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(raw), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return -1;
  auto kern = q4k_gemv_tma_kernel<NP, NST, XP>;
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024),
                         "cudaFuncSetAttribute(q4k tma smem)");
    if (rc) return rc;
    rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                     "cudaFuncSetAttribute(q4k tma cluster)");
    if (rc) return rc;
    configured_dev = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.cs, (a.N + kRows - 1) / kRows, (a.M + a.mchunk - 1) / a.mchunk);
  if constexpr (XP) {
    // stage the activations once: one CTA per token row, chunks of kXpTokens tokens
    const XSrc xsrc{a.x, nullptr, nullptr, a.ldx, a.x_dtype, a.x_vec, a.M, 0};
    prestage_x3_kernel<8, 32, 256, kXpTokens, 1><<<a.M, 256, 0, st>>>(xsrc, a.K, const_cast<uint8_t*>(a.xg),
                                                                      a.chunk_bytes, a.sum_off);
    const int rc = cuda_status(cudaGetLastError(), "q4k prestage launch");
    if (rc) return rc;
  }
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
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, tm, a), "q4k_gemv_tma launch");
}

}  // namespace

// Bytes of the global activation staging of an M-token call (0 up to 4 tokens).
size_t q4k_stage_workspace(int M, int K) {
  if (M <= 4) return 0;
  const long sum_off = (long)K * gemv::xb3_slots(kXpTokens);
  const long chunk = (sum_off + (long)(K / kBlkVals) * q4k_sum_ints(kXpTokens) * 4 + 255) & ~255L;
  return (size_t)((M + kXpTokens - 1) / kXpTokens) * (size_t)chunk;
}

// Returns true (and the launch status in *rc) when the TMA-fed kernel takes this call.
// Up to 4 tokens: one z-slice that stages its own activations; more: activations staged once in
// global memory (the caller's workspace when large enough, else the stream-ordered allocator),
// z-slices of 8 tokens. The cluster size is chosen so the CTAs fill whole resident waves of the
// SMs as evenly as possible, two CTAs per SM where they fit.
bool q4k_gemv_tma(const void* x, int x_dtype, long ldx, const uint8_t* raw, const float* bias, void* out,
                  int out_dtype, long ldo, int M, int K, int N, cudaStream_t st, int* rc, void* workspace,
                  size_t ws_bytes) {
  static int enabled = -1, sms = 0;
  if (enabled < 0) {
    enabled = env_int("QL_Q4K_TMA", 1);
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  if (!enabled || M <= 0) return false;
  Q4kTmaArgs a = {};
  a.x = x; a.ldx = ldx; a.x_dtype = x_dtype;
  const int vec_elems = x_dtype == QL_F32 ? 4 : 8;
  a.x_vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (ldx % vec_elems == 0);
  a.bias = bias; a.out = out; a.ldo = ldo; a.out_dtype = out_dtype;
  a.M = M; a.K = K; a.N = N;
  a.nb = K / kBlkVals;
  const bool xp = M > 4;
  const int mchunk = xp ? kXpTokens : M;
  a.mchunk = mchunk;
  a.xsize = x_dtype == QL_F32 ? 4 : 2;
  a.pdl = (launch_flags() & QL_LAUNCH_PDL) ? 1 : 0;
  a.xbulk = !xp && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (ldx * a.xsize) % 16 == 0;
  const int xbs = a.xbulk ? a.xsize : 0;
  const int zdim = (M + mchunk - 1) / mchunk;
  const int tiles = (N + kRows - 1) / kRows * zdim;
  const size_t per_sm = 228 * 1024;   // shared memory per SM; each CTA also reserves 1 KB
  int best_cs = 0, best_nst = kNST;
  double best = -1.0;
  for (int ns = kNST; ns >= 2; ns -= 2) {   // ring depths built: 4 and 2
    for (int c = 1; c <= 8 && c <= a.nb; ++c) {
      const size_t sm = smem_bytes(mchunk, a.nb, c, ns, xp, xbs);
      if (sm > 220 * 1024) continue;
      const int fit = (int)(per_sm / (sm + 1024 + 256));
      const int per = fit >= 2 ? 2 : fit;
      if (per < 1) continue;
      const int slots = sms * per;
      const int ctas = tiles * c;
      if (ctas > slots && c > 1) continue;
      const double waves = (double)ctas / slots;
      const double busiest = (double)((ctas + slots - 1) / slots);
      double score = waves / busiest * (ctas < slots ? (double)ctas / slots : 1.0);
      if (per < 2) score *= 0.75;
      if (score > best + 1e-9) {
        best = score;
        best_cs = c;
        best_nst = ns;
      }
    }
  }
  if (best_cs == 0) return false;
  a.cs = best_cs;
  a.nst = best_nst;
  const size_t smem = smem_bytes(mchunk, a.nb, a.cs, a.nst, xp, xbs);
  void* ws = nullptr;
  bool owned = false;
  if (xp) {
    // per chunk: B operand of all K (K * slots bytes), then one sums record per super-block
    a.sum_off = (long)K * gemv::xb3_slots(kXpTokens);
    a.chunk_bytes = (a.sum_off + (long)a.nb * q4k_sum_ints(kXpTokens) * 4 + 255) & ~255L;
    const size_t need = q4k_stage_workspace(M, K);
    if (workspace && ws_bytes >= need) {
      ws = workspace;
    } else {
      const int arc = stream_alloc(&ws, need, st, "ql_q4k_matmul: staging");
      if (arc) {
        *rc = arc;
        return true;
      }
      owned = true;
    }
    a.xg = reinterpret_cast<const uint8_t*>(ws);
  }
  int r;
  if (xp) {
    r = a.nst == kNST ? launch<4, kNST, true>(a, raw, smem, st) : launch<4, 2, true>(a, raw, smem, st);
    if (owned) {
      const int frc = cuda_status(cudaFreeAsync(ws, st), "cudaFreeAsync(q4k staging)");
      if (r == 0) r = frc;
    }
    if (r < 0) {   // declined after the staging ran: report, the register kernel would redo it
      set_error("ql_q4k_matmul: tensor-map encoding failed");
      r = QL_ERR_CUDA;
    }
  } else if (M <= 2) {
    r = a.nst == kNST ? launch<1, kNST, false>(a, raw, smem, st) : launch<1, 2, false>(a, raw, smem, st);
  } else {
    r = a.nst == kNST ? launch<2, kNST, false>(a, raw, smem, st) : launch<2, 2, false>(a, raw, smem, st);
  }
  if (r < 0) return false;
  *rc = r;
  return true;
}

}  // namespace ql
