// GPTQ decode GEMV, TMA-fed: one producer warp streams the packed weights, their scales and
// their zero points through a shared-memory ring with tensor-memory-accelerator (TMA) copies,
// so each CTA keeps its whole ring in flight however long the consumer warps take per stage;
// consumer warps touch only shared memory.
//
// Arithmetic: integer tensor-core MMA (mma.sync m16n8k32, u8 weights x s8 activation bytes).
// An int4 word (8 consecutive K of one column) becomes two A-fragment registers with three ALU
// ops; an int8 word is an A register as it is. Activations are staged as 23-bit integers with one
// power-of-two exponent per group (gemv_common.cuh, stage_x3), split into three signed byte
// planes that occupy three MMA columns per token. Per group the MMA yields exact int32 dot
// products, and the zero point folds into the group sums S of the staged integers:
//   acc += scale * 2^e * (C - (z + off) * S),   C = 256 * C_hi + C_lo (exact)
// for the lane that owns the (b2, b1) plane pair and for the lane that owns (b0, 0); the two
// lanes' sums are added (the first times 2^8) when the kernel finishes.
//
// Ring stage = 128 values of K for the CTA's 256 (or 128) columns:
//   weights  3-D TMA box over the packed weight viewed as [N/32 strips][K/per rows][32 columns]:
//            per 32-column strip a [rows][128 B] block with the 128-byte swizzle (16-byte chunk
//            c of row r at chunk c ^ (r % 8)); consumer warp w reads strip w % SW, lane (g, t) of
//            step s the 16 bytes of row 4s + t, chunk g (at most 2-way bank conflicts)
//   scales   2-D box [groups of the stage][tile columns]
//   zeros    2-D box [groups of the stage][tile columns / per words]
// Split-K runs over a thread-block cluster; partial sums go to the owning rank's shared memory.
#include <cooperative_groups.h>
#include <cuda.h>

#include "gemv_common.cuh"
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

constexpr int kCW = 8;                 // consumer warps
constexpr int kThreads = (kCW + 1) * 32;
constexpr int kStageK = 128;           // K per ring stage
// A CTA covers SW 32-column strips (tile of 32 * SW columns); its kCW consumer warps are
// SW strips x KW = kCW / SW ways along K (K-way j consumes the stages i with i % KW == j).
// SW = 8 suits wide layers; SW = 4 doubles the CTAs of narrow ones so every SM gets two.

struct TmaGemvArgs {
  const void* x;
  const int32_t* x_rows;   // NULL, or the x row of each output row (MoE token gather)
  const int32_t* x_perm;
  long ldx;
  int x_dtype;
  int x_vec;
  int sc_dtype;
  const float* bias;
  void* out;
  long ldo;
  int out_dtype;
  int M, K, N, gs;
  int nstage;   // K / kStageK
  int cs;       // cluster size along K
  int sw;       // 32-column strips per CTA (8 or 4; host-side choice)
  int nst;      // ring stages (the kernel's NST; host-side choice)
  float zoff;
  // grouped (MoE) mode when g_offsets != NULL: blockIdx.z is an entry of the device-built tile
  // table (expert e = g_tiles[2z], first row g_tiles[2z + 1] of its segment, MAXM rows at
  // most); the expert's weights start at packed row e * g_wrows and group row e * g_grows
  const int32_t* g_offsets;
  const int32_t* g_tiles;
  const int32_t* g_n_tiles;
  int g_wrows, g_grows;
  int g_max_tiles;  // host: table capacity (grid z)
  int n_experts;    // host: stacked weight matrices (1 when dense)
  int glu;          // > 0: x rows are [gate | up] glu elements apart (SwiGLU applied when staging)
  // dense calls of up to 4 tokens whose rows of x are 16-byte aligned (no gather): the producer
  // copies the CTA's slice of x into shared memory with bulk copies ahead of the weights, so the
  // consumers' staging reads shared memory instead of queueing behind the weight stream
  int xbulk;
  int xsize;      // bytes per element of x
  int pdl;        // launched as a programmatic dependent (x copies wait for the previous kernel)
  // fused decode-step options (dense calls): RMSNorm of each token row over all K folded into
  // the staging (norm_w [K], with xbulk the whole rows are copied), and a residual added to the
  // output (res [M, ldres] fp32; may alias out: every element is read and written by one thread)
  const float* norm_w;
  float norm_eps;
  const float* res;
  long ldres;
  // dense calls of more than 4 tokens: activations staged once in global memory, blockIdx.z
  // taking tokens [z * MAXM, z * MAXM + MAXM) from chunk z at xg + z * xg_chunk (the B operand
  // of all K, then per group [S1 | S0 | fe][MAXM] at xg_sum_off)
  const uint8_t* xg;
  long xg_chunk, xg_sum_off;
};

// Activation source of one CTA (its rows of x, possibly gathered).
struct XSrc {
  const void* x;
  const int32_t* x_rows;
  const int32_t* x_perm;
  long ldx;
  int x_dtype;
  int x_vec;
  int M;
  int glu;   // > 0: rows are [gate | up] glu elements apart; the activation is silu(gate) * up
  const float* nw;   // RMSNorm weight [K] folded into the loads (NULL: none)
  const float* nr;   // per-token factor 1 / sqrt(mean(x^2) + eps), indexed by token
  float norm_eps;
};

// Ring stage: weights, scales, zeros; with XP also the stage's B operand (4 steps x 4 lanes x
// kXSlots slots x 8 bytes) and its group sums [GPS][3][MAXM]. MAXM = 2 NP tokens (NP MMA tiles).
template <int BITS, int GS, int NST, int SCB, int SW, int MAXM = 2, bool XP = false>
struct TmaLayout {
  static constexpr int PER = 32 / BITS;
  static constexpr int TC = 32 * SW;                       // columns per CTA tile
  static constexpr int GPS = kStageK / GS;                 // groups per stage (>= 1)
  static constexpr int ROWS = kStageK / PER;               // packed rows per stage
  static constexpr int kStripBytes = ROWS * 128;
  static constexpr int kWBytes = SW * kStripBytes;         // 2 KB per strip (int4) / 4 KB (int8)
  static constexpr int kScBytes = GPS * TC * SCB;          // scales of the stage
  static constexpr int kZBytes = GPS * (TC / PER) * 4;
  static constexpr int kWSZBytes = (kWBytes + kScBytes + kZBytes + 15) & ~15;
  static constexpr int kXSlots = gemv::xb3_slots(MAXM);
  static constexpr int kXBytes = XP ? kStageK * kXSlots : 0;
  static constexpr int kGBytes = XP ? GPS * 3 * MAXM * 4 : 0;
  static constexpr int kStageBytes = (kWSZBytes + kXBytes + kGBytes + 1023) & ~1023;
  static constexpr int kBarOff = NST * kStageBytes;
  static constexpr int kXsOff = kBarOff + 2 * NST * 8 + 32;   // + abort flag, reduction and x barriers
};

// NP MMA tiles of two tokens each (MAXM = 2 NP tokens per CTA).
template <int BITS, int GS, int NP, int NST, int SCB, int SW, bool XP>
__global__ void __launch_bounds__(kThreads, 2)
    gptq_gemv_tma_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_s,
                         const __grid_constant__ CUtensorMap tmap_z, const TmaGemvArgs a) {
  constexpr int MAXM = 2 * NP;
  using L = TmaLayout<BITS, GS, NST, SCB, SW, MAXM, XP>;
  constexpr int TC = L::TC;
  constexpr int KW = kCW / SW;
  constexpr int PER = L::PER;
  constexpr int GPS = L::GPS;
  constexpr int SPG = GS / 32;                             // 32-K MMA steps per group
  constexpr uint32_t MASK = (1u << BITS) - 1u;
  static_assert(KW == 1 || NST % 2 == 0, "two K-ways need an even ring depth (each slot stays with one way)");

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = ptx::smem_addr(smem);
  const uint32_t bar_full = sbase + L::kBarOff;
  const uint32_t bar_empty = bar_full + 8 * NST;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kBarOff + 16 * NST);
  const uint32_t bar_red = bar_full + 16 * NST + 8;   // partial sums received from the cluster
  const uint32_t bar_x = bar_full + 16 * NST + 16;    // the bulk copy of x (xbulk)

  // which rows this CTA takes: grouped mode reads the tile table (uniform over the cluster,
  // which shares blockIdx.z; slots without rows leave before any barrier), dense calls of more
  // than MAXM tokens take token chunk z
  int M = a.M, e = 0;
  long row0 = 0;
  if (a.g_offsets) {
    // the table is written by the routing kernel: under programmatic dependent launch it can be
    // read only once that kernel has completed (this CTA's weights depend on it anyway)
    pdl_wait();
    const int tz = blockIdx.z;
    if (tz >= *a.g_n_tiles) return;
    e = a.g_tiles[2 * tz];
    row0 = a.g_offsets[e] + a.g_tiles[2 * tz + 1];
    M = min(MAXM, a.g_offsets[e + 1] - (int)row0);
  } else if (XP) {
    row0 = (long)blockIdx.z * MAXM;
    M = min(MAXM, a.M - (int)row0);
  }
  const uint8_t* xgc = XP ? a.xg + (long)blockIdx.z * a.xg_chunk : nullptr;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int rank = blockIdx.x;
  const int sq = a.nstage / a.cs, srem = a.nstage - sq * a.cs;
  const int s0 = rank * sq + min(rank, srem);
  const int nst = sq + (rank < srem ? 1 : 0);
  const int klen = nst * kStageK;
  const int nst_max = sq + (srem ? 1 : 0);
  const int klen_max = nst_max * kStageK;
  const int ng_max = nst_max * GPS;
  const int N = a.N;
  // staged activations (without XP): B rows of sstride slots, then [3 M rows][gstride] ints of
  // group sums and factors (row 3m: S of v1, 3m + 1: S of b0, 3m + 2: fe bits)
  const int sstride = XP ? L::kXSlots : gemv::xb3_slots(M);
  const int gstride = ng_max | 1;
  uint2* xb = reinterpret_cast<uint2*>(smem + L::kXsOff);
  const int xs_bytes = XP ? 0 : (klen_max * sstride + 15) & ~15;
  int* gsum = reinterpret_cast<int*>(smem + L::kXsOff + xs_bytes);
  const int gs_bytes = XP ? 0 : (3 * M * gstride * 4 + 15) & ~15;
  // xbulk: the raw rows of x for this CTA's K slice, klen_max elements apart (with the RMSNorm
  // option the whole rows, K apart: the norm needs every element)
  unsigned char* xraw = smem + L::kXsOff + xs_bytes + gs_bytes;
  const int xr_ld = a.norm_w ? a.K : klen_max;            // elements between token rows
  const int xr_k0 = a.norm_w ? 0 : s0 * kStageK;          // first element copied
  const int xr_len = a.norm_w ? a.K : klen;               // elements copied per row
  const int xr_bytes = a.xbulk ? (M * xr_ld * a.xsize + 15) & ~15 : 0;
  float* red = reinterpret_cast<float*>(smem + L::kXsOff + xs_bytes + gs_bytes + xr_bytes);
  // red: [cs ranks][MAXM tokens][cq_max * 4 columns], cs * cq_max <= Q + cs - 1, cs <= 16 (only
  // with cs > 1); kred: K-way partials (KW == 2), [SW * 32 lanes][NP * 4]
  float* kred = red + (a.cs > 1 ? (TC + 64) * MAXM : 0);

  // Split-K reduction over the cluster: rank q owns the column quads [qs(q), qs(q + 1)) of
  // the tile, qs(q) = ceil(q * Q / cs), Q = TC / 4; every rank sends each owner its partial
  // sums for the owner's columns with 16-byte st.async stores that count down the owner's
  // mbarrier, so each CTA waits only for the partials it reduces.
  constexpr int Q = TC / 4;
  const int cs = a.cs;
  const int cq_max = (Q + cs - 1) / cs;                     // column quads per owner (max)
  const int oq0 = (rank * Q + cs - 1) / cs, oq1 = ((rank + 1) * Q + cs - 1) / cs;
  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, SW);
    }
    ptx::mbar_init(bar_red, 1);
    ptx::mbar_init(bar_x, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    if (cs > 1) ptx::mbar_arrive_expect_tx(bar_red, (uint32_t)(cs * M * (oq1 - oq0) * 16));
  }
  __syncthreads();
  if (cs > 1) cluster_arrive_relaxed();   // waited for before the first remote store

  // the bulk copy of this CTA's x slice (one copy per token row)
  auto copy_x = [&]() {
    pdl_wait();   // x may be the previous kernel's output
    const uint32_t row_bytes = (uint32_t)(xr_len * a.xsize);
    ptx::mbar_arrive_expect_tx(bar_x, (uint32_t)M * row_bytes);
    const char* xs = reinterpret_cast<const char*>(a.x) + (size_t)xr_k0 * a.xsize;
    for (int m = 0; m < M; ++m)
      ptx::bulk_load(ptx::smem_addr(xraw + (size_t)m * xr_ld * a.xsize), xs + (size_t)(row0 + m) * a.ldx * a.xsize,
                     row_bytes, bar_x);
  };

  if (warp == kCW) {
    // ------------------------------------------------------------ producer warp
    if (lane == 0) {
      ptx::tma_prefetch(&tmap_w);
      ptx::tma_prefetch(&tmap_s);
      ptx::tma_prefetch(&tmap_z);
      const int strip0 = blockIdx.y * SW;
      const int wrow0 = e * a.g_wrows, grow0 = e * a.g_grows;   // expert's first rows (0 when dense)
      if (XP) pdl_wait();   // the staged activations are the previous kernel's output
      // x goes first into the memory queue, unless this grid may start before the previous
      // kernel ends: then the weights (independent of it) go first and x after the ring's fill
      const bool x_first = a.xbulk && !a.pdl;
      const int x_after = a.xbulk && a.pdl ? min(NST, nst) - 1 : -1;
      if (x_first) copy_x();
      int i = 0;
      bool ok = true;
      for (; i < nst; ++i) {
        const int s = i % NST;
        if (i == NST) pdl_trigger();
        if (!ptx::mbar_wait(bar_empty + 8 * s, ((i / NST) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t st = sbase + s * L::kStageBytes;
        const uint32_t fb = bar_full + 8 * s;
        const int srow = grow0 + ((s0 + i) * kStageK) / a.gs;   // first scale/zero row of the stage
        ptx::mbar_arrive_expect_tx(fb, L::kWBytes + L::kScBytes + L::kZBytes + L::kXBytes + L::kGBytes);
        asm volatile(
            "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
            "[%2];" ::"r"(st),
            "l"(reinterpret_cast<uint64_t>(&tmap_w)), "r"(fb), "r"(0), "r"(wrow0 + (s0 + i) * L::ROWS), "r"(strip0)
            : "memory");
        ptx::tma_load_2d(st + L::kWBytes, &tmap_s, fb, blockIdx.y * TC, srow);
        ptx::tma_load_2d(st + L::kWBytes + L::kScBytes, &tmap_z, fb, blockIdx.y * (TC / PER), srow);
        if constexpr (XP) {
          ptx::bulk_load(st + L::kWSZBytes, xgc + (long)(s0 + i) * L::kXBytes, L::kXBytes, fb);
          ptx::bulk_load(st + L::kWSZBytes + L::kXBytes, xgc + a.xg_sum_off + (long)(s0 + i) * L::kGBytes, L::kGBytes,
                         fb);
        }
        if (i == x_after) copy_x();
      }
      if (nst <= NST) pdl_trigger();
      if (!ok) {
        for (int j = i > NST ? i - NST : 0; j < i; ++j) ptx::mbar_wait_drain(bar_full + 8 * (j % NST), (j / NST) & 1);
        if (x_first || (x_after >= 0 && i > x_after)) ptx::mbar_wait_drain(bar_x, 0);
      }
    }
    __syncwarp();
    if (cs > 1) cluster_wait_acquire();   // pairs with the arrive above (every thread once)
  } else {
    // ------------------------------------------------------------ consumer warps
    // Lane (g, t) owns columns 4g .. 4g+3 of its warp's 32-column strip. MMA m16n8k32: rows
    // g / g + 8 of tile 0 are columns 4g / 4g + 1, of tile 1 columns 4g + 2 / 4g + 3. In MMA
    // tile mq, B columns 4u .. 4u + 3 hold b2, b1, 0, b0 of token 2 mq + u, so the lane's D
    // columns 2t, 2t + 1 are the plane pair t % 2 ((b2, b1) or (0, b0)) of token 2 mq + t / 2
    // and C = 256 * D[2t] + D[2t + 1] is the exact dot product with v1 or with b0.
    const int gq = lane >> 2, t = lane & 3;
    const int strip = warp % SW, kway = warp / SW;
    const int lcol = strip * 32 + gq * 4;                   // first of this lane's 4 columns
    const int c0 = blockIdx.y * TC + lcol;
    const bool col_ok = c0 < N;
    const int zoff = (int)a.zoff;
    const int ptok = t >> 1, pp = t & 1;                     // D side: token in tile, plane pair
    // B side: token in tile, and the stored plane of column gq (columns 4u .. 4u + 3 of token
    // u are b2, b1, zero, b0, so that the lane pairs read (b2, b1) and (0, b0))
    const int btok = gq >> 2, bpl = (gq & 3) == 3 ? 2 : (gq & 3);
    const bool bld = (gq & 3) != 2;
    pdl_wait();   // x may be the previous kernel's output
    bool x_ok = true;
    if constexpr (!XP) {
      auto sums = [&](int m, int g, int s1, int s0v) {
        gsum[(3 * m) * gstride + g] = s1;
        gsum[(3 * m + 1) * gstride + g] = s0v;
      };
      auto expo = [&](int m, int g, float fe) { gsum[(3 * m + 2) * gstride + g] = __float_as_int(fe); };
      if (a.xbulk) x_ok = ptx::mbar_wait(bar_x, 0, abort_flag);   // x arrives in shared memory by bulk copy
      // this CTA's rows: the bulk copy, or x itself (gathered through x_rows, else from row row0 on)
      const size_t x_off = a.x_rows ? 0 : (size_t)row0 * (size_t)a.ldx * (a.x_dtype == QL_F32 ? 4u : 2u);
      XSrc xsrc = a.xbulk ? XSrc{xraw, nullptr, nullptr, xr_ld, a.x_dtype, 1, M, 0}
                          : XSrc{reinterpret_cast<const char*>(a.x) + x_off, a.x_rows ? a.x_rows + row0 : nullptr,
                                 a.x_perm, a.ldx, a.x_dtype, a.x_vec, M, a.glu};
      if (a.norm_w) {
        // RMSNorm: each token row's 1 / sqrt(mean(x^2) + eps) over all K, then x * r * w on load
        __shared__ float sh_nr[4], sh_red[kCW][4];
        for (int m = 0; m < M; ++m) {
          float ss = x_ok ? gemv::row_sumsq_part(xsrc, m, a.K, tid, kCW * 32) : 0.f;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          if (lane == 0) sh_red[warp][m] = ss;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kCW * 32) : "memory");
        if (tid < M) {
          float t = 0.f;
          for (int w = 0; w < kCW; ++w) t += sh_red[w][tid];
          sh_nr[tid] = rsqrtf(t / (float)a.K + a.norm_eps);
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kCW * 32) : "memory");
        xsrc.nw = a.norm_w;
        xsrc.nr = sh_nr;
      }
      const int kb = a.xbulk && !a.norm_w ? 0 : s0 * kStageK;   // the slice's first K in xsrc
      gemv::stage_x3<BITS, GS, GS, true>(xsrc, kb, x_ok ? klen : 0, sstride, xb, sums, expo, tid, kCW * 32);
    }

    float acc[NP][4];
#pragma unroll
    for (int mq = 0; mq < NP; ++mq)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[mq][c] = 0.f;

    const uint32_t strip_off = strip * L::kStripBytes;
    const uint32_t xb_base = ptx::smem_addr(xb);
    for (int i = kway; i < (x_ok ? nst : 0); i += KW) {
      const int s = i % NST;
      if (!ptx::mbar_wait(bar_full + 8 * s, (i / NST) & 1, abort_flag)) break;
      const uint32_t st = sbase + s * L::kStageBytes;
      const unsigned char* stp = smem + s * L::kStageBytes;
#pragma unroll
      for (int u = 0; u < GPS; ++u) {
        int d[NP][2][4];
#pragma unroll
        for (int mq = 0; mq < NP; ++mq)
#pragma unroll
          for (int p = 0; p < 2; ++p)
#pragma unroll
            for (int q = 0; q < 4; ++q) d[mq][p][q] = 0;
#pragma unroll
        for (int sp = 0; sp < SPG; ++sp) {
          const int step = (i * GPS + u) * SPG + sp;                // 32-K step inside the slice
          uint32_t A0[4], A1[4];                                    // tile 0 / tile 1 A registers
          if constexpr (BITS == 4) {
            const int row = (u * SPG + sp) * 4 + t;                 // packed row inside the stage
            const uint32_t addr = st + strip_off + row * 128 + ((gq ^ (row & 7)) << 4);
            uint4 w;
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
                         : "r"(addr));
            // even K offsets of each word -> bytes of register 0, odd -> register 1
            A0[0] = w.x & 0x0F0F0F0Fu; A0[1] = w.y & 0x0F0F0F0Fu;
            A0[2] = (w.x >> 4) & 0x0F0F0F0Fu; A0[3] = (w.y >> 4) & 0x0F0F0F0Fu;
            A1[0] = w.z & 0x0F0F0F0Fu; A1[1] = w.w & 0x0F0F0F0Fu;
            A1[2] = (w.z >> 4) & 0x0F0F0F0Fu; A1[3] = (w.w >> 4) & 0x0F0F0F0Fu;
          } else {
            const int r0 = (u * SPG + sp) * 8 + t, r1 = r0 + 4;
            const uint32_t ad0 = st + strip_off + r0 * 128 + ((gq ^ (r0 & 7)) << 4);
            const uint32_t ad1 = st + strip_off + r1 * 128 + ((gq ^ (r1 & 7)) << 4);
            uint4 w, v;
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
                         : "r"(ad0));
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                         : "r"(ad1));
            A0[0] = w.x; A0[1] = w.y; A0[2] = v.x; A0[3] = v.y;
            A1[0] = w.z; A1[1] = w.w; A1[2] = v.z; A1[3] = v.w;
          }
#pragma unroll
          for (int mq = 0; mq < NP; ++mq) {
            const int tok = 2 * mq + btok;
            uint32_t b0 = 0u, b1 = 0u;
            if (bld && tok < M) {
              const uint32_t xa = XP ? st + L::kWSZBytes + (((u * SPG + sp) * 4 + t) * sstride + 3 * tok + bpl) * 8
                                     : xb_base + ((step * 4 + t) * sstride + 3 * tok + bpl) * 8;
              asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(xa));
            }
            mma_16832_u8s8(d[mq][0], A0[0], A0[1], A0[2], A0[3], b0, b1);
            mma_16832_u8s8(d[mq][1], A1[0], A1[1], A1[2], A1[3], b0, b1);
          }
        }
        // fold the group: acc += scale * 2^e * (C - (z + off) * S), C = 256 * C_hi + C_lo (exact)
        const int gl = i * GPS + u;
        float scv[4];
        if constexpr (SCB == 2) {
          const uint2 h = *reinterpret_cast<const uint2*>(stp + L::kWBytes + (u * TC + lcol) * 2);
          if (a.sc_dtype == QL_BF16) {
            scv[0] = __uint_as_float(h.x << 16); scv[1] = __uint_as_float(h.x & 0xffff0000u);
            scv[2] = __uint_as_float(h.y << 16); scv[3] = __uint_as_float(h.y & 0xffff0000u);
          } else {
            const float2 f0 = __half22float2(u32_as_h2(h.x)), f1 = __half22float2(u32_as_h2(h.y));
            scv[0] = f0.x; scv[1] = f0.y; scv[2] = f1.x; scv[3] = f1.y;
          }
        } else {
          const float4 f = *reinterpret_cast<const float4*>(stp + L::kWBytes + (u * TC + lcol) * 4);
          scv[0] = f.x; scv[1] = f.y; scv[2] = f.z; scv[3] = f.w;
        }
        const uint32_t zw = *reinterpret_cast<const uint32_t*>(stp + L::kWBytes + L::kScBytes +
                                                               (u * (TC / PER) + lcol / PER) * 4) >>
                            (BITS * (lcol % PER));
        int zo[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) zo[c] = (int)((zw >> (BITS * c)) & MASK) + zoff;
#pragma unroll
        for (int mq = 0; mq < NP; ++mq) {
          const int tok = 2 * mq + ptok;
          int S = 0;
          float fe = 0.f;
          if (tok < M) {
            if constexpr (XP) {
              const int* gsr = reinterpret_cast<const int*>(stp + L::kWSZBytes + L::kXBytes) + u * 3 * MAXM;
              S = gsr[pp * MAXM + tok];
              fe = __int_as_float(gsr[2 * MAXM + tok]);
            } else {
              S = gsum[(3 * tok + pp) * gstride + gl];
              fe = __int_as_float(gsum[(3 * tok + 2) * gstride + gl]);
            }
          }
          const int C[4] = {d[mq][0][0] * 256 + d[mq][0][1], d[mq][0][2] * 256 + d[mq][0][3],
                            d[mq][1][0] * 256 + d[mq][1][1], d[mq][1][2] * 256 + d[mq][1][3]};
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[mq][c] = fmaf(scv[c] * fe, (float)(C[c] - zo[c] * S), acc[mq][c]);
        }
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_empty + 8 * s);
    }

    if constexpr (KW == 2) {
      // the second K-way hands its partial sums to the first through shared memory
      float* kr = kred + (strip * 32 + lane) * (NP * 4);
      if (kway == 1) {
#pragma unroll
        for (int mq = 0; mq < NP; ++mq)
#pragma unroll
          for (int c = 0; c < 4; ++c) kr[mq * 4 + c] = acc[mq][c];
      }
      asm volatile("bar.sync 2, %0;" ::"r"(kCW * 32) : "memory");
      if (kway == 0) {
#pragma unroll
        for (int mq = 0; mq < NP; ++mq)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[mq][c] += kr[mq * 4 + c];
      }
    }
    // the (b2, b1) lane's sums count 2^8 times the (b0, 0) lane's; add the pair (exact scaling)
#pragma unroll
    for (int mq = 0; mq < NP; ++mq)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float v = pp ? acc[mq][c] : 256.f * acc[mq][c];
        acc[mq][c] = v + __shfl_xor_sync(0xffffffffu, v, 1);
      }
    const bool writer = kway == 0 && pp == 0;
    if (cs == 1) {
#pragma unroll
      for (int mq = 0; mq < NP; ++mq) {
        const int tok = 2 * mq + ptok;
        if (writer && tok < M && col_ok) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float v = acc[mq][c];
            if (a.bias) v += a.bias[c0 + c];
            if (a.res) v += a.res[(row0 + tok) * a.ldres + c0 + c];
            store_from_float(a.out, a.out_dtype, (row0 + tok) * a.ldo + c0 + c, v);
          }
        }
      }
    } else {
      __syncwarp();
      cluster_wait_acquire();   // every CTA of the cluster has initialised its mbarriers
      if (writer) {
        const int lq = lcol >> 2;
        const int owner = (lq * cs) / Q;
        const int oq = (owner * Q + cs - 1) / cs;
        const uint32_t rbase = ptx::mapa(ptx::smem_addr(red), owner);
        const uint32_t rbar = ptx::mapa(bar_red, owner);
#pragma unroll
        for (int mq = 0; mq < NP; ++mq) {
          const int tok = 2 * mq + ptok;
          if (tok < M) {
            const uint32_t dst = rbase + (((rank * MAXM + tok) * cq_max + (lq - oq)) * 4) * 4;
            ptx::st_async_v4(dst, acc[mq][0], acc[mq][1], acc[mq][2], acc[mq][3], rbar);
          }
        }
      }
    }
  }

  if (cs > 1) {
    // reduce the owned columns over the ranks in rank order (deterministic) and store
    const bool got = ptx::mbar_wait(bar_red, 0, abort_flag);
    const int ncol = (oq1 - oq0) * 4;
    if (got) {
      for (int s = tid; s < ncol * M; s += blockDim.x) {
        const int tok = s / ncol, c = s - tok * ncol;
        float v = 0.f;
        for (int q = 0; q < cs; ++q) v += red[(q * MAXM + tok) * cq_max * 4 + c];
        const int col = blockIdx.y * TC + oq0 * 4 + c;
        if (col < N) {
          if (a.bias) v += a.bias[col];
          if (a.res) v += a.res[(row0 + tok) * a.ldres + col];
          store_from_float(a.out, a.out_dtype, (row0 + tok) * a.ldo + col, v);
        }
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

bool encode_2d(EncodeTiledFn enc, CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
               uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

constexpr int kMaxSmem = 220 * 1024;

// Ring depth (NST) of the kernel built for (bits, sw): the same bytes in flight for both tile
// widths. Batches of more than 2 tokens that stage their activations per CTA may also take a ring
// of half that depth, so that two CTAs with their larger activation slices still fit on one SM.
// With two K-ways (sw < kCW) the ring depth must be even: way j consumes the stages i with
// i % 2 == j, and an even depth keeps every ring slot with one way. With an odd depth the two ways
// alternate on a slot, so a way that runs ahead can wait on a slot two phases early, find the
// barrier parity it waits for already set, and read a stage that has not been refilled.
constexpr int nst_cap(int bits, int sw) { return (bits == 4 ? 4 : 3) * (kCW / sw); }
constexpr int nst_half(int bits, int sw) {
  return sw < kCW ? (nst_cap(bits, sw) / 2 >= 4 ? (nst_cap(bits, sw) / 2) & ~1 : 2)
                  : (nst_cap(bits, sw) / 2 > 2 ? nst_cap(bits, sw) / 2 : 2);
}

// MMA tiles (two tokens each) of a CTA that takes m tokens.
constexpr int np_of(int m) { return m <= 2 ? 1 : (m <= 4 ? 2 : 4); }
constexpr int kXpTokens = 8;   // tokens per CTA when the activations are staged in global memory

// Dynamic shared memory of one CTA (ring of nst = NST stages) that takes m tokens, as the
// kernel's prologue carves it up: 1 KB of alignment slack, the ring, the barriers, the staged
// activations and their group sums / factors (unless xp: then each stage carries its own), the
// raw slice of x when it arrives by bulk copy (xbulk_size = bytes per element, else 0), the
// split-K receive buffer (cs > 1) and the K-way hand-off (128-column tiles).
size_t tma_smem(int bits, int kgs, int scb, int sw, int nst, int cs, int m, int nstage, bool xp, int xbulk_size = 0,
                bool xbulk_full_rows = false) {
  const int per = 32 / bits, tc = 32 * sw, gps = kStageK / kgs, rows = kStageK / per;
  const int np = xp ? kXpTokens / 2 : np_of(m), maxm = 2 * np;
  const size_t wsz = ((size_t)sw * rows * 128 + (size_t)gps * tc * scb + (size_t)gps * (tc / per) * 4 + 15) & ~(size_t)15;
  const size_t xpart = xp ? (size_t)kStageK * gemv::xb3_slots(maxm) + (size_t)gps * 3 * maxm * 4 : 0;
  const size_t stage = (wsz + xpart + 1023) & ~(size_t)1023;
  const int sq = nstage / cs, nst_max = sq + (nstage % cs ? 1 : 0);
  const int ng_max = nst_max * gps;
  size_t b = 1024 + (size_t)nst * stage + 2 * nst * 8 + 16;
  if (!xp) {
    b += ((size_t)nst_max * kStageK * gemv::xb3_slots(m) + 15) & ~(size_t)15;
    b += ((size_t)3 * m * (ng_max | 1) * 4 + 15) & ~(size_t)15;
    if (xbulk_size)
      b += ((size_t)m * (xbulk_full_rows ? (size_t)nstage * kStageK : (size_t)nst_max * kStageK) * xbulk_size + 15) &
           ~(size_t)15;
  }
  if (cs > 1) b += (size_t)(tc + 64) * maxm * 4;
  if (sw < kCW) b += (size_t)sw * 32 * np * 4 * 4;
  return b;
}

template <int BITS, int GS, int NP, int NST, int SCB, int SW, bool XP>
int launch_tma(const TmaGemvArgs& a, const uint32_t* qweight, const uint32_t* qzeros, const void* scales,
               cudaStream_t st) {
  using L = TmaLayout<BITS, GS, NST, SCB, SW, 2 * NP, XP>;
  constexpr int TC = L::TC;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return -1;
  CUtensorMap tw, ts, tz;
  {
    const cuuint64_t dims[3] = {32, (cuuint64_t)a.n_experts * (a.K / L::PER), (cuuint64_t)(a.N / 32)};
    const cuuint64_t strides[2] = {(cuuint64_t)a.N * 4, 128};
    const cuuint32_t box[3] = {32, (cuuint32_t)L::ROWS, (cuuint32_t)SW};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (enc(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint32_t*>(qweight), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return -1;
  }
  const int G = a.K / a.gs;
  const CUtensorMapDataType sdt = SCB == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                           : (a.sc_dtype == QL_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  if (!encode_2d(enc, &ts, sdt, scales, a.N, (uint64_t)a.n_experts * G, (uint64_t)a.N * SCB, TC, L::GPS)) return -1;
  if (!encode_2d(enc, &tz, CU_TENSOR_MAP_DATA_TYPE_UINT32, qzeros, a.N / L::PER, (uint64_t)a.n_experts * G,
                 (uint64_t)(a.N / L::PER) * 4,
                 TC / L::PER, L::GPS))
    return -1;
  auto kern = gptq_gemv_tma_kernel<BITS, GS, NP, NST, SCB, SW, XP>;
  const size_t smem = tma_smem(BITS, GS, SCB, SW, NST, a.cs, XP ? kXpTokens : a.M, a.nstage, XP,
                              a.xbulk ? a.xsize : 0, a.norm_w != nullptr);
  if (smem > kMaxSmem) return -1;  // too large an activation slice: caller falls back
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem),
                         "cudaFuncSetAttribute(tma gemv smem)");
    if (rc) return rc;
    rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                     "cudaFuncSetAttribute(tma gemv cluster)");
    if (rc) return rc;
    configured_dev = dev;
  }
  cudaLaunchConfig_t cfg = {};
  const int zdim = a.g_offsets ? a.g_max_tiles : (XP ? (a.M + kXpTokens - 1) / kXpTokens : 1);
  cfg.gridDim = dim3(a.cs, (a.N + TC - 1) / TC, zdim);
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
  if constexpr (XP) {
    // stage the activations once (one CTA per token row) for every CTA of the GEMV
    const XSrc xsrc{a.x, nullptr, a.x_perm, a.ldx, a.x_dtype, a.x_vec, a.M, a.glu, a.norm_w, nullptr, a.norm_eps};
    prestage_x3_kernel<BITS, GS, GS, kXpTokens, 0><<<a.M, 256, 0, st>>>(xsrc, a.K, const_cast<uint8_t*>(a.xg),
                                                                       a.xg_chunk, a.xg_sum_off);
    const int rc = cuda_status(cudaGetLastError(), "gptq prestage launch");
    if (rc) return rc;
  }
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, tw, ts, tz, a), "gptq_gemv_tma launch");
}

template <int BITS, int GS, int SW, int SCB>
int tma_np(const TmaGemvArgs& a, const uint32_t* qw, const uint32_t* qz, const void* sc, cudaStream_t st) {
  constexpr int CAP = nst_cap(BITS, SW), HALF = nst_half(BITS, SW);
  if (a.xg)   // activations staged in global memory: full ring, no staging area
    return launch_tma<BITS, GS, 4, CAP, SCB, SW, true>(a, qw, qz, sc, st);
  if (a.M <= 2) return launch_tma<BITS, GS, 1, CAP, SCB, SW, false>(a, qw, qz, sc, st);
  if (a.M <= 4)
    return a.nst == CAP ? launch_tma<BITS, GS, 2, CAP, SCB, SW, false>(a, qw, qz, sc, st)
                        : launch_tma<BITS, GS, 2, HALF, SCB, SW, false>(a, qw, qz, sc, st);
  return a.nst == CAP ? launch_tma<BITS, GS, 4, CAP, SCB, SW, false>(a, qw, qz, sc, st)
                      : launch_tma<BITS, GS, 4, HALF, SCB, SW, false>(a, qw, qz, sc, st);
}

template <int BITS, int GS>
int tma_mt(const TmaGemvArgs& a, const uint32_t* qw, const uint32_t* qz, const void* sc, cudaStream_t st) {
  if (a.sc_dtype == QL_F32)
    return a.sw == 8 ? tma_np<BITS, GS, 8, 4>(a, qw, qz, sc, st) : tma_np<BITS, GS, 4, 4>(a, qw, qz, sc, st);
  return a.sw == 8 ? tma_np<BITS, GS, 8, 2>(a, qw, qz, sc, st) : tma_np<BITS, GS, 4, 2>(a, qw, qz, sc, st);
}

template <int BITS>
int tma_gs(const TmaGemvArgs& a, int kgs, const uint32_t* qw, const uint32_t* qz, const void* sc, cudaStream_t st) {
  switch (kgs) {
    case 32: return tma_mt<BITS, 32>(a, qw, qz, sc, st);
    case 64: return tma_mt<BITS, 64>(a, qw, qz, sc, st);
    default: return tma_mt<BITS, 128>(a, qw, qz, sc, st);
  }
}

// Tile width (a.sw), cluster size (a.cs, the K split) and ring depth (a.nst) for CTAs of m
// tokens: the CTA count tiles * zdim * cs should fill resident waves of the SMs as evenly as
// possible, two CTAs per SM where their shared memory allows (a shallower ring is preferred to a
// single CTA per SM); the wider tile and the deeper ring win ties.
void choose_split(TmaGemvArgs& a, int N, int m, int zdim, int sms, int ctas_per_sm, int max_cluster, int bits,
                  int kgs, int scb, bool xp) {
  int cs = 1, sw = 8, nst = nst_cap(bits, 8);
  double best = -1.0;
  const size_t per_sm = 228 * 1024;   // shared memory per SM; each CTA also reserves 1 KB
  for (int w = 8; w >= 4; w /= 2) {
    const int tiles = (N + 32 * w - 1) / (32 * w) * zdim;
    const int cap = nst_cap(bits, w), half = nst_half(bits, w);
    for (int ns = cap; ns >= half; ns = (ns == cap && m > 2 && half < cap && !xp) ? half : 0) {
      for (int c = 1; c <= max_cluster && c <= 16 && c <= a.nstage; ++c) {
        const size_t sm = tma_smem(bits, kgs, scb, w, ns, c, m, a.nstage, xp, a.xbulk ? a.xsize : 0,
                                   a.norm_w != nullptr);
        if (sm > (size_t)kMaxSmem) continue;
        const int fit = (int)(per_sm / (sm + 1024 + 256));
        const int per = fit < ctas_per_sm ? fit : ctas_per_sm;
        if (per < 1) continue;
        const int slots = sms * per;
        const int ctas = tiles * c;
        if (ctas > slots && c > 1) continue;
        const double waves = (double)ctas / slots;
        const double busiest = (double)((ctas + slots - 1) / slots);
        double score = waves / busiest * (ctas < slots ? (double)ctas / slots : 1.0);
        if (per < ctas_per_sm) score *= 0.75;
        if (score > best + 1e-9) {
          best = score;
          cs = c;
          sw = w;
          nst = ns;
        }
      }
    }
  }
  a.sw = sw;
  a.cs = cs;
  a.nst = nst;
}

// Bytes of one token chunk of the global staging (B operand of all K, then the group sums and
// factors), 256-byte aligned.
size_t stage_chunk_bytes(int K, int kgs) {
  const size_t body = (size_t)K * gemv::xb3_slots(kXpTokens) + (size_t)(K / kgs) * 3 * kXpTokens * 4;
  return (body + 255) & ~(size_t)255;
}

}  // namespace

// Bytes of global staging a dense call of M tokens needs (0 when it stages in shared memory):
// one chunk per kXpTokens tokens.
size_t gemv_stage_workspace(int M, int K, int kgs) {
  if (M <= 4 || M > 16) return 0;
  return (size_t)((M + kXpTokens - 1) / kXpTokens) * stage_chunk_bytes(K, kgs);
}

// Returns true (and the launch status in *rc) when the TMA-fed GEMV handles this shape.
// Dense GEMV of M <= 16 tokens. More than 4 tokens: the activations are staged once in global
// memory (the caller's workspace when it is large enough, else the stream-ordered allocator).
bool gptq_gemv_tma(const void* x, int x_dtype, long ldx, const int32_t* x_perm, const int32_t* qweight,
                   const int32_t* qzeros, const void* scales, int sc_dtype, const float* bias, void* out,
                   int out_dtype, long ldo, int M, int K, int N, int gs, int bits, float zoff, cudaStream_t st,
                   int* rc, void* workspace, size_t ws_bytes, const GemvFused* fu) {
  static int enabled = -1, sms = 0, ctas_per_sm = 0, max_cluster = 8;
  if (enabled < 0) {
    enabled = env_int("QL_GEMV_TMA", 1);
    ctas_per_sm = env_int("QL_GEMV_TMA_CTAS_PER_SM", 2);
    // clusters of 16 CTAs with this kernel's shared memory do not all fit in one wave
    max_cluster = env_int("QL_GEMV_MAX_CLUSTER", 8);
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  if (!enabled || M > 16 || N % 32 != 0 || K % kStageK != 0 || (gs % 128 != 0 && gs != 32 && gs != 64)) return false;
  if ((reinterpret_cast<uintptr_t>(qweight) & 15) || (reinterpret_cast<uintptr_t>(qzeros) & 15) ||
      (reinterpret_cast<uintptr_t>(scales) & 15))
    return false;
  const int kgs = gs % 128 == 0 ? 128 : gs;
  TmaGemvArgs a = {};
  a.n_experts = 1;
  a.x = x; a.x_rows = nullptr; a.x_perm = x_perm; a.ldx = ldx; a.x_dtype = x_dtype;
  const int vec_elems = x_dtype == QL_F32 ? 4 : 8;
  a.x_vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (ldx % vec_elems == 0);
  a.sc_dtype = sc_dtype; a.bias = bias;
  a.out = out; a.ldo = ldo; a.out_dtype = out_dtype;
  a.M = M; a.K = K; a.N = N; a.gs = gs; a.zoff = zoff;
  a.nstage = K / kStageK;
  if (fu) {
    a.norm_w = fu->norm_w; a.norm_eps = fu->norm_eps; a.glu = fu->glu; a.res = fu->res; a.ldres = fu->ldres;
  }
  const size_t need = gemv_stage_workspace(M, K, kgs);
  void* ws = nullptr;
  bool owned = false;
  if (need) {
    if (workspace && ws_bytes >= need) {
      ws = workspace;
    } else {
      const int arc = stream_alloc(&ws, need, st, "ql_gptq_matmul: decode staging");
      if (arc) {
        *rc = arc;
        return true;
      }
      owned = true;
    }
    a.xg = reinterpret_cast<const uint8_t*>(ws);
    a.xg_chunk = (long)stage_chunk_bytes(K, kgs);
    a.xg_sum_off = (long)K * gemv::xb3_slots(kXpTokens);
  }
  const int zdim = need ? (M + kXpTokens - 1) / kXpTokens : 1;
  a.xsize = x_dtype == QL_F32 ? 4 : 2;
  a.pdl = (launch_flags() & QL_LAUNCH_PDL) ? 1 : 0;
  a.xbulk = !need && x_perm == nullptr && !a.glu && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
            (ldx * a.xsize) % 16 == 0;
  choose_split(a, N, need ? kXpTokens : M, zdim, sms, ctas_per_sm, max_cluster, bits, kgs, sc_dtype == QL_F32 ? 4 : 2,
               need != 0);
  const uint32_t* qw = reinterpret_cast<const uint32_t*>(qweight);
  const uint32_t* qz = reinterpret_cast<const uint32_t*>(qzeros);
  int r = bits == 4 ? tma_gs<4>(a, kgs, qw, qz, scales, st) : tma_gs<8>(a, kgs, qw, qz, scales, st);
  if (owned) {
    const int frc = cuda_status(cudaFreeAsync(ws, st), "cudaFreeAsync(gemv staging)");
    if (r == 0) r = frc;
  }
  if (r < 0) {
    if (!need) return false;
    set_error("ql_gptq_matmul: tensor-map encoding failed");   // after the staging ran
    r = QL_ERR_CUDA;
  }
  *rc = r;
  return true;
}

// Grouped (MoE) form: one launch over the tiles of a device-built table (tile_rows = 4 or 8
// rows of one expert per tile) for stacked weights (qweight [E][K/per][N], qzeros
// [E][K/gs][N/per], scales [E][K/gs][N]); output row p of expert e's sorted rows is
// x[x_rows[p]] (x[p] when x_rows is NULL) @ W_e.
bool gptq_gemv_tma_grouped(const void* x, int x_dtype, long ldx, const int32_t* x_rows, const int32_t* qweight,
                           const int32_t* qzeros, const void* scales, int sc_dtype, int E, const int32_t* offsets,
                           const int32_t* tiles, const int32_t* n_tiles, int max_tiles, int tile_rows, void* out,
                           int out_dtype, long ldo, int K, int N, int gs, int bits, float zoff, cudaStream_t st,
                           int* rc, int glu) {
  int sms = 148, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (env_int("QL_GEMV_TMA", 1) == 0 || N % 32 != 0 || K % kStageK != 0 || (gs % 128 != 0 && gs != 32 && gs != 64))
    return false;
  if ((tile_rows != 4 && tile_rows != 8) || !tiles || !n_tiles || max_tiles <= 0) return false;
  if ((reinterpret_cast<uintptr_t>(qweight) & 15) || (reinterpret_cast<uintptr_t>(qzeros) & 15) ||
      (reinterpret_cast<uintptr_t>(scales) & 15))
    return false;
  const int kgs = gs % 128 == 0 ? 128 : gs;
  const int per = 32 / bits;
  TmaGemvArgs a = {};
  a.x = x; a.x_rows = x_rows; a.x_perm = nullptr; a.ldx = ldx; a.x_dtype = x_dtype;
  const int vec_elems = x_dtype == QL_F32 ? 4 : 8;
  a.x_vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (ldx % vec_elems == 0);
  a.sc_dtype = sc_dtype; a.bias = nullptr;
  a.out = out; a.ldo = ldo; a.out_dtype = out_dtype;
  a.M = tile_rows;   // rows per tile (selects NP, sizes smem)
  a.K = K; a.N = N; a.gs = gs; a.zoff = zoff;
  a.nstage = K / kStageK;
  a.g_offsets = offsets; a.g_tiles = tiles; a.g_n_tiles = n_tiles;
  a.g_max_tiles = max_tiles;
  a.glu = glu;
  a.g_wrows = K / per;
  a.g_grows = K / gs;
  a.n_experts = E;
  choose_split(a, N, a.M, max_tiles, sms, 2, 8, bits, kgs, sc_dtype == QL_F32 ? 4 : 2, false);
  const uint32_t* qw = reinterpret_cast<const uint32_t*>(qweight);
  const uint32_t* qz = reinterpret_cast<const uint32_t*>(qzeros);
  const int r = bits == 4 ? tma_gs<4>(a, kgs, qw, qz, scales, st) : tma_gs<8>(a, kgs, qw, qz, scales, st);
  if (r < 0) return false;
  *rc = r;
  return true;
}

}  // namespace ql

// ---------------------------------------------------------------------------------------
// fused decode-step linear
// ---------------------------------------------------------------------------------------
extern "C" int ql_gptq_matmul_fused(const void* x, int x_dtype, long ldx, const int32_t* x_perm,
                                    const int32_t* qweight, const int32_t* qzeros, const void* scales,
                                    int scales_dtype, const float* bias, const float* norm_weight, float norm_eps,
                                    int glu, const float* residual, long ld_residual, void* out, int out_dtype,
                                    long ldo, int M, int K, int N, int gs, int bits, float zero_offset,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  using namespace ql;
  if (bits != 4 && bits != 8) {
    set_error("ql_gptq_matmul_fused: bits must be 4 or 8 (got %d)", bits);
    return QL_ERR_UNSUPPORTED;
  }
  const int per = 32 / bits;
  if (M < 0 || K <= 0 || N <= 0 || gs <= 0 || K % gs || K % per || N % per || ldo < N ||
      ldx < (glu ? 2L * K : (long)K) || (glu && glu != K) || (residual && ld_residual < N) ||
      (x_dtype != QL_F32 && x_dtype != QL_F16 && x_dtype != QL_BF16) ||
      (out_dtype != QL_F32 && out_dtype != QL_F16 && out_dtype != QL_BF16) ||
      (scales_dtype != QL_F32 && scales_dtype != QL_F16 && scales_dtype != QL_BF16) ||
      (zero_offset != 0.f && zero_offset != 1.f)) {
    set_error("ql_gptq_matmul_fused: bad arguments (M=%d K=%d N=%d gs=%d glu=%d ldx=%ld)", M, K, N, gs, glu, ldx);
    return QL_ERR_ARG;
  }
  if (norm_weight && glu) {
    set_error("ql_gptq_matmul_fused: the RMSNorm and SwiGLU prologues do not combine");
    return QL_ERR_UNSUPPORTED;
  }
  if (M == 0) return QL_OK;
  if (!x || !qweight || !qzeros || !scales || !out) {
    set_error("ql_gptq_matmul_fused: null pointer");
    return QL_ERR_ARG;
  }
  if (M > 16) {
    set_error("ql_gptq_matmul_fused: decode-step path, M=%d > 16 (use ql_gptq_matmul)", M);
    return QL_ERR_UNSUPPORTED;
  }
  const GemvFused fu{norm_weight, norm_eps, glu, residual, ld_residual};
  int rc = QL_OK;
  if (!gptq_gemv_tma(x, x_dtype, ldx, x_perm, qweight, qzeros, scales, scales_dtype, bias, out, out_dtype, ldo, M, K,
                     N, gs, bits, zero_offset, (cudaStream_t)stream, &rc, workspace, workspace_bytes, &fu)) {
    set_error("ql_gptq_matmul_fused: shape outside the fused GEMV (N %% 32 == 0, K %% 128 == 0, gs 32 / 64 / "
              "multiple of 128, 16-byte aligned weights)");
    return QL_ERR_UNSUPPORTED;
  }
  return rc;
}
