// GPTQ int4/int8 prefill dequant-GEMM on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// y[M, N] = x[M, K] @ W[K, N], W = scales[g, n] * (q[k, n] - (z[g, n] + zero_offset)).
//
// The product is computed transposed, D^T[n, m] = W^T[n, :] . x^T[:, m], so that
//  * the dequantised weights are the MMA's A operand held in tensor memory: 8 dequant warps
//    (two per TMEM lane quadrant, each taking half of a 64-K slab) own one output column per
//    lane, unpack the packed words in registers and write fp16 straight into TMEM with
//    tcgen05.st;
//  * the activations are the B operand: a 128-token x 64-k fp16 tile per stage, 128-byte
//    swizzled;
//  * one TMA producer warp streams every operand of a slab into a shared-memory ring: the
//    activation tile, the packed weight box [rows of the slab][128 columns], and the slab's
//    scale and zero rows, so no compute warp ever waits on a global load;
//  * the fp32 accumulator (128 columns x 128 tokens) is double-buffered in TMEM: epilogue warps
//    drain one buffer with tcgen05.ld while the MMAs of the next tile fill the other.
//
// Numerics: the MMA runs in fp16 with fp32 accumulation. x is staged once (prep_x_kernel) as
// fp16 scaled per row by an exact power of two (largest |x| in [2^14, 2^15)), which keeps
// fp16's 11-bit significand for bf16/fp32 inputs without overflow; the weights are
// fp16(scale * (q - z - off)), one rounding of 2^-12 relative. The staging also applies the
// act-order permutation x[:, perm[k]] and stores each 8-value block in the (j, j+4) pair order
// that the register unpack produces, so weights and activations agree on K order.
//
// Warp roles (512 threads, one CTA per SM, persistent over output tiles):
//   warp 0       TMA producer
//   warp 1       TMEM allocator and MMA issuer (one elected lane)
//   warps 4-11   dequant producers (TMEM lane quadrant = warp % 4, slab half = (warp - 4) / 4)
//   warps 12-15  epilogue (TMEM lanes 0-127)
#include <cuda.h>
#include <cudaTypedefs.h>


#include "ql_common.cuh"
#include "sm100_ptx.cuh"

namespace ql {

// device-side status of the tensor-core kernels (a bounded wait that gave up)
__device__ int g_tc_status = 0;

namespace {

constexpr int kSlabK = 64;          // K per pipeline stage
constexpr int kTileN = 128;         // output columns per tile (MMA M, TMEM lanes)
constexpr int kBT = 128;            // tokens per tile (MMA N)
constexpr int kThreads = 512;
constexpr int kDequantWarp0 = 4;
constexpr int kDequantWarps = 8;
constexpr int kEpilogueWarp0 = 12;
constexpr int kFmtGptq = 0;          // packed GPTQ words + scale and zero rows (AutoGPTQ layout)
constexpr int kFmtQ4K = 1;           // GGUF Q4_K super-blocks read in place: 144 bytes / 256 values
constexpr int kQ4kBlockBytes = 144;

// ---------------------------------------------------------------------------------------
// activation staging: fp16, power-of-two row scale, act-order gather, (j, j+4) pair order
// ---------------------------------------------------------------------------------------
// Position of value j of an 8-value block in the staging: int4 words pair (j, j+4) of each
// 8-block, int8 words pair (j, j+2) of each 4-block (the order the register unpack produces).
template <int BITS>
__device__ __forceinline__ int pair_pos(int j) {
  return BITS == 4 ? (j & 3) * 2 + (j >> 2) : (j & 4) + (j & 1) * 2 + ((j >> 1) & 1);
}

// Largest |value| of a 16-byte vector of x_dtype elements.
__device__ __forceinline__ float absmax16(uint4 u, int x_dtype) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (x_dtype == QL_F32) {
      m = fmaxf(m, fabsf(__uint_as_float(w[i])));
    } else if (x_dtype == QL_BF16) {
      m = fmaxf(m, fmaxf(fabsf(__uint_as_float(w[i] << 16)), fabsf(__uint_as_float(w[i] & 0xffff0000u))));
    } else {
      const float2 f = __half22float2(u32_as_h2(w[i]));
      m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
  return m;
}

constexpr int kPrepSmemMax = 96 * 1024;   // rows up to this many bytes are staged through smem

// SwiGLU of element k of a fused [gate | up] row y[base .. base + 2K): silu(g) * u with
// silu(v) = v / (1 + e^-v), the expression of the MoE activation kernel (_core.py:502-503).
__device__ __forceinline__ float swiglu_at(const void* y, int y_dtype, long base, int k, int K) {
  const float g = load_as_float(y, y_dtype, base + k);
  const float u = load_as_float(y, y_dtype, base + K + k);
  return g / (1.0f + expf(-g)) * u;
}

// One CTA per row: the row is copied into shared memory with 16-byte loads (taking the row
// maximum on the way), then gathered through the act-order permutation from shared memory.
// With glu (== K) the row is a fused [gate | up] row of 2K values and the staged value is their
// SwiGLU, formed once into shared memory as fp32.
template <int BITS>
__global__ void __launch_bounds__(256) prep_x_kernel(const void* __restrict__ x, int x_dtype, long ldx,
                                                     const int32_t* __restrict__ perm,
                                                     const int32_t* __restrict__ row_map, int M, int K, int glu,
                                                     __half* __restrict__ x16, int* __restrict__ row_exp) {
  extern __shared__ __align__(16) unsigned char xrow[];
  __shared__ float wmax[8];
  __shared__ int sh_e;
  const int m = blockIdx.x;
  const int tid = threadIdx.x;
  const int esz = x_dtype == QL_F32 ? 4 : 2;
  const long row = row_map ? row_map[m] : m;   // row_map: MoE token gather
  const unsigned char* src = reinterpret_cast<const unsigned char*>(x) + (size_t)row * ldx * esz;
  float mx = 0.f;
  if (glu) {
    float* arow = reinterpret_cast<float*>(xrow);
    if (x_dtype == QL_F32 && (reinterpret_cast<uintptr_t>(src) & 15) == 0 && K % 4 == 0) {
      const float4* g4 = reinterpret_cast<const float4*>(src);
      const float4* u4 = g4 + K / 4;
      for (int i = tid; i < K / 4; i += blockDim.x) {
        const float4 g = g4[i], u = u4[i];
        const float a0 = g.x / (1.0f + expf(-g.x)) * u.x, a1 = g.y / (1.0f + expf(-g.y)) * u.y;
        const float a2 = g.z / (1.0f + expf(-g.z)) * u.z, a3 = g.w / (1.0f + expf(-g.w)) * u.w;
        reinterpret_cast<float4*>(arow)[i] = make_float4(a0, a1, a2, a3);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(a0), fabsf(a1)), fmaxf(fabsf(a2), fabsf(a3))));
      }
    } else {
      for (int k = tid; k < K; k += blockDim.x) {
        const float v = swiglu_at(x, x_dtype, row * ldx, k, K);
        arow[k] = v;
        mx = fmaxf(mx, fabsf(v));
      }
    }
  } else if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {   // K * esz is a multiple of 128 (K % 64 == 0)
    for (int i = tid; i < K * esz / 16; i += blockDim.x) {
      const uint4 u = reinterpret_cast<const uint4*>(src)[i];
      reinterpret_cast<uint4*>(xrow)[i] = u;
      mx = fmaxf(mx, absmax16(u, x_dtype));
    }
  } else {
    for (int k = tid; k < K; k += blockDim.x) {
      const float v = load_as_float(x, x_dtype, row * ldx + k);
      if (esz == 4) reinterpret_cast<float*>(xrow)[k] = v;
      else reinterpret_cast<uint16_t*>(xrow)[k] = reinterpret_cast<const uint16_t*>(src)[k];
      mx = fmaxf(mx, fabsf(v));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) wmax[tid >> 5] = mx;
  __syncthreads();
  if (tid == 0) {
    float v = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) v = fmaxf(v, wmax[i]);
    sh_e = stage_exponent(v);
    row_exp[m] = sh_e;
  }
  __syncthreads();
  const float s = exp2i(-sh_e);
  const int row_dtype = glu ? QL_F32 : x_dtype;
  for (int b = tid; b < K / 8; b += blockDim.x) {
    __align__(16) __half h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = b * 8 + j;
      const int srck = perm ? perm[k] : k;
      h[pair_pos<BITS>(j)] = __float2half_rn(load_as_float(xrow, row_dtype, srck) * s);
    }
    *reinterpret_cast<uint4*>(x16 + (long)m * K + b * 8) = *reinterpret_cast<uint4*>(h);
  }
}

// The same for rows larger than kPrepSmemMax: gathers straight from global memory.
template <int BITS>
__global__ void __launch_bounds__(256) prep_x_global_kernel(const void* __restrict__ x, int x_dtype, long ldx,
                                                            const int32_t* __restrict__ perm,
                                                            const int32_t* __restrict__ row_map, int M, int K,
                                                            int glu, __half* __restrict__ x16,
                                                            int* __restrict__ row_exp) {
  __shared__ float wmax[8];
  __shared__ int sh_e;
  const int m = blockIdx.x;
  const int tid = threadIdx.x;
  const long base = (long)(row_map ? row_map[m] : m) * ldx;
  float mx = 0.f;
  for (int k = tid; k < K; k += blockDim.x)
    mx = fmaxf(mx, fabsf(glu ? swiglu_at(x, x_dtype, base, k, K) : load_as_float(x, x_dtype, base + k)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) wmax[tid >> 5] = mx;
  __syncthreads();
  if (tid == 0) {
    float v = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) v = fmaxf(v, wmax[i]);
    sh_e = stage_exponent(v);
    row_exp[m] = sh_e;
  }
  __syncthreads();
  const float s = exp2i(-sh_e);
  for (int b = tid; b < K / 8; b += blockDim.x) {
    __align__(16) __half h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = b * 8 + j;
      const int src = perm ? perm[k] : k;
      const float v = glu ? swiglu_at(x, x_dtype, base, src, K) : load_as_float(x, x_dtype, base + src);
      h[pair_pos<BITS>(j)] = __float2half_rn(v * s);
    }
    *reinterpret_cast<uint4*>(x16 + (long)m * K + b * 8) = *reinterpret_cast<uint4*>(h);
  }
}

// Launch the activation staging for M rows.
int launch_prep_x(int bits, const void* x, int x_dtype, long ldx, const int32_t* perm, const int32_t* row_map, int M,
                  int K, __half* x16, int* row_exp, cudaStream_t st, int glu = 0) {
  const size_t bytes = (size_t)K * (glu || x_dtype == QL_F32 ? 4 : 2);
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    int rc = cuda_status(cudaFuncSetAttribute(prep_x_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              kPrepSmemMax),
                         "cudaFuncSetAttribute(prep_x)");
    if (!rc)
      rc = cuda_status(cudaFuncSetAttribute(prep_x_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            kPrepSmemMax),
                       "cudaFuncSetAttribute(prep_x)");
    if (rc) return rc;
    configured_dev = dev;
  }
  if (bytes <= (size_t)kPrepSmemMax) {
    if (bits == 4)
      prep_x_kernel<4><<<M, 256, bytes, st>>>(x, x_dtype, ldx, perm, row_map, M, K, glu, x16, row_exp);
    else
      prep_x_kernel<8><<<M, 256, bytes, st>>>(x, x_dtype, ldx, perm, row_map, M, K, glu, x16, row_exp);
  } else if (bits == 4) {
    prep_x_global_kernel<4><<<M, 256, 0, st>>>(x, x_dtype, ldx, perm, row_map, M, K, glu, x16, row_exp);
  } else {
    prep_x_global_kernel<8><<<M, 256, 0, st>>>(x, x_dtype, ldx, perm, row_map, M, K, glu, x16, row_exp);
  }
  return cuda_status(cudaGetLastError(), "prep_x launch");
}

// ---------------------------------------------------------------------------------------
// GEMM
// ---------------------------------------------------------------------------------------
struct GemmArgs {
  const uint32_t* qw;
  const uint32_t* qz;
  const void* sc;
  int sc_dtype;
  const float* bias;
  const int* row_exp;
  void* out;
  long ldo;
  int out_dtype;
  int M, K, N, gs;
  float zoff;
  int n_wtiles, n_ttiles;
  int gb;            // scale/zero rows per slab: 2 when gs == 32, else 1
  // grouped (MoE) mode when tiles != NULL: token tile i is rows [offsets[e] + r, offsets[e + 1])
  // capped at BT rows, with (e, r) = tiles[2i], tiles[2i + 1]; *n_tiles tiles are valid
  const int32_t* tiles;
  const int32_t* n_tiles;
  const int32_t* offsets;
  long qw_estride, qz_estride, sc_estride;
};

// Rows of token tile `tt` and the expert whose weights it uses.
struct TileRows {
  int row0, row_end, e;
};
__device__ __forceinline__ TileRows tile_rows(const GemmArgs& a, int tt, int BT) {
  TileRows r;
  if (a.tiles) {
    r.e = a.tiles[2 * tt];
    r.row0 = a.offsets[r.e] + a.tiles[2 * tt + 1];
    r.row_end = a.offsets[r.e + 1];
  } else {
    r.e = 0;
    r.row0 = tt * BT;
    r.row_end = a.M;
  }
  return r;
}

// A stage covers SK values of K (64 or 128): SK / 64 activation boxes of [BT rows][64 K] fp16
// (128-byte swizzled rows, one box after the other), the packed weights of those K, one or two
// scale / zero rows. Q4_K stages hold the 64 quant bytes of each row's half super-block ([128][64],
// 64-byte swizzled) and the rows' 16-byte block headers (d, dmin, scales).
template <int BITS, int NS, int BT, int SK = kSlabK, int FMT = kFmtGptq>
struct SmemLayout {
  static constexpr int PER = 32 / BITS;
  static constexpr int ROWS = SK / PER;                    // packed rows per stage (8 / 16 int4)
  static constexpr int kXBytes = BT * SK * 2;              // activation boxes, 128-byte swizzled rows
  static constexpr int kWOff = kXBytes;
  // packed weights [ROWS][128] words, or (Q4_K) [128 rows][64 quant bytes]
  static constexpr int kWBytes = FMT == kFmtQ4K ? kTileN * 64 : ROWS * kTileN * 4;
  static constexpr int kSOff = kWOff + kWBytes;
  // scales [<= 2 groups][128], or (Q4_K) the rows' block headers [128][16 bytes]
  static constexpr int kSBytes = FMT == kFmtQ4K ? kTileN * 16 : 2 * kTileN * 4;
  static constexpr int kZOff = kSOff + kSBytes;
  static constexpr int kZBytes = FMT == kFmtQ4K ? 0 : 2 * (kTileN / PER) * 4;   // zeros [<= 2][128 / PER]
  static constexpr int kStageBytes = (kZOff + kZBytes + 1023) & ~1023;
  static constexpr int kBarOff = NS * kStageBytes;
  // barriers: full[NS] (activations), a_full[NS], slab_free[NS], d_full[2], d_empty[2], final,
  // w_full[NS] (packed weights, scales, zeros)
  static constexpr int kNumBars = 4 * NS + 5;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kEpiOff = (kMiscOff + 16 + 15) & ~15;   // after the tmem slot and abort flag
  static constexpr int kEpiBytes = 4 * 32 * 32 * 4;           // epilogue transpose, [32][32] fp32 a warp
  static constexpr int kBytes = kEpiOff + kEpiBytes + 1024;   // + alignment slack
};

// Unpack one packed int4 word (8 values along K) for one column into 4 fp16 pairs
// (q_j, q_{j+4}) * scale; q - z - off is exact in fp16 before the single scale rounding.
__device__ __forceinline__ void dq_int4(uint32_t w, uint32_t zlo, uint32_t zhi, __half2 s2, uint32_t* out4) {
  const __half2 one16 = __floats2half2_rn(0.0625f, 0.0625f);
  const uint32_t w8 = w >> 8;
  const uint32_t v0 = lop3_andor(w, 0x000F000Fu, kMagicF16x2);
  const uint32_t v1 = lop3_andor(w, 0x00F000F0u, kMagicF16x2);
  const uint32_t v2 = lop3_andor(w8, 0x000F000Fu, kMagicF16x2);
  const uint32_t v3 = lop3_andor(w8, 0x00F000F0u, kMagicF16x2);
  out4[0] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(v0), u32_as_h2(zlo)), s2));
  out4[1] = h2_as_u32(__hmul2(__hfma2(u32_as_h2(v1), one16, u32_as_h2(zhi)), s2));
  out4[2] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(v2), u32_as_h2(zlo)), s2));
  out4[3] = h2_as_u32(__hmul2(__hfma2(u32_as_h2(v3), one16, u32_as_h2(zhi)), s2));
}
// int8: one word = 4 values along K -> pairs (q0, q2), (q1, q3)
__device__ __forceinline__ void dq_int8(uint32_t w, uint32_t zlo, __half2 s2, uint32_t* out2) {
  const uint32_t v0 = lop3_andor(w, 0x00FF00FFu, kMagicF16x2);
  const uint32_t v1 = lop3_andor(w >> 8, 0x00FF00FFu, kMagicF16x2);
  out2[0] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(v0), u32_as_h2(zlo)), s2));
  out2[1] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(v1), u32_as_h2(zlo)), s2));
}

// BT = tokens per tile (MMA N). Up to 128 two accumulators sit in TMEM at columns 0 and 128 (the
// epilogue drains one while the next tile's MMAs fill the other): 128 for dense GEMMs, 32 / 64 for
// MoE experts with few rows each (less padding, same dequant work per tile). BT = 256 halves the
// dequant work per MMA flop with one accumulator (the next tile waits for the drain).
// SK = K per pipeline stage (64, or 128 for dense GEMMs with whole 128-value groups): a larger
// stage halves every role's per-stage handshakes (barrier waits, TMEM-store waits, commits).
template <int BITS, int NS, int BT, int SK, bool DQ_ALT_T, int FMT>
__global__ void __launch_bounds__(kThreads, 1)
    gptq_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_s, const __grid_constant__ CUtensorMap tmap_z,
                        const GemmArgs a) {
  using L = SmemLayout<BITS, NS, BT, SK, FMT>;
  static_assert(FMT == kFmtGptq || (BITS == 4 && SK == 2 * kSlabK && DQ_ALT_T), "Q4_K: 128-value stages");
  constexpr int PER = L::PER;
  constexpr int ROWS = L::ROWS;
  constexpr int HROWS = ROWS / 2;               // packed rows per dequant half
  constexpr int TCOLS_A = SK / 2;               // TMEM columns per A stage (fp16 pairs)
  static_assert(SK == kSlabK || SK == 2 * kSlabK || SK == 4 * kSlabK, "stage K");
  static_assert(BT == 32 || BT == 64 || BT == 128, "token tile");
  static_assert(!DQ_ALT_T || NS % 2 == 0, "alternating dequant groups: a stage's previous use is the group's own");
  constexpr int ND = 2;                         // accumulator buffers
  constexpr int DCOL = BT;                      // TMEM columns between accumulator buffers
  constexpr int A_COL = ND * DCOL;              // A stages start after the accumulators
  constexpr bool DQ_ALT = DQ_ALT_T;               // dequant groups on alternate stages
  constexpr uint32_t IDESC = ptx::idesc_f16_f32(kTileN, BT);
  constexpr uint32_t MASK = (1u << BITS) - 1u;
  static_assert(A_COL + NS * TCOLS_A <= 512, "TMEM budget");

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // the 128-byte swizzle pattern is anchored to 1024-byte boundaries
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = ptx::smem_addr(smem);
  const uint32_t bar0 = sbase + L::kBarOff;
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto a_full = [&](int s) { return bar0 + 8u * (NS + s); };
  auto slab_free = [&](int s) { return bar0 + 8u * (2 * NS + s); };
  auto d_full = [&](int b) { return bar0 + 8u * (3 * NS + b); };
  auto d_empty = [&](int b) { return bar0 + 8u * (3 * NS + 2 + b); };
  const uint32_t fin_bar = bar0 + 8u * (3 * NS + 4);
  auto w_full = [&](int s) { return bar0 + 8u * (3 * NS + 5 + s); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      ptx::mbar_init(full(s), 1);
      ptx::mbar_init(w_full(s), 1);
      ptx::mbar_init(a_full(s), DQ_ALT ? kDequantWarps / 2 : kDequantWarps);
      ptx::mbar_init(slab_free(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(d_full(b), 1);
      ptx::mbar_init(d_empty(b), 128);
    }
    ptx::mbar_init(fin_bar, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_addr(tmem_slot), 512);
    ptx::tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    ptx::tma_prefetch(&tmap_x);
    ptx::tma_prefetch(&tmap_w);
    ptx::tma_prefetch(&tmap_s);
    ptx::tma_prefetch(&tmap_z);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int nslab = a.K / SK;
  const int ntiles = a.n_wtiles * (a.tiles ? *a.n_tiles : a.n_ttiles);
  const int G = a.K / a.gs;
  const int sc_bytes = a.sc_dtype == QL_F32 ? 4 : 2;

  if (warp == 0) {
    // ---------------- TMA producer: activation tile, packed weights, scales, zeros per slab
    if (lane == 0) {
      // the weight side of a stage has its own barrier so the dequant warps start on it while the
      // (four times larger) activation tile is still in flight
      const uint32_t w_tx = FMT == kFmtQ4K ? (uint32_t)(L::kWBytes + L::kSBytes)
                                           : L::kWBytes + a.gb * kTileN * sc_bytes + a.gb * (kTileN / PER) * 4;
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
        const int wt = tile % a.n_wtiles;
        const TileRows tr = tile_rows(a, tile / a.n_wtiles, BT);
        const int wrow0 = tr.e * (a.K / PER), grow0 = tr.e * G;
        for (int kb = 0; kb < nslab; ++kb, ++it) {
          const int s = it % NS;
          if (!ptx::mbar_wait_sleep(slab_free(s), ((it / NS) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t st = sbase + s * L::kStageBytes;
          const int g0 = (kb * SK) / a.gs;
          ptx::mbar_arrive_expect_tx(w_full(s), w_tx);
          if constexpr (FMT == kFmtQ4K) {
            // quant bytes of half kb & 1 of super-block kb / 2, and the block headers (x = byte
            // offset in the row)
            const int xb0 = (kb >> 1) * kQ4kBlockBytes;
            ptx::tma_load_2d(st + L::kWOff, &tmap_w, w_full(s), xb0 + 16 + 64 * (kb & 1), wt * kTileN);
            ptx::tma_load_2d(st + L::kSOff, &tmap_s, w_full(s), xb0, wt * kTileN);
          } else {
            ptx::tma_load_2d(st + L::kWOff, &tmap_w, w_full(s), wt * kTileN, wrow0 + kb * ROWS);
            ptx::tma_load_2d(st + L::kSOff, &tmap_s, w_full(s), wt * kTileN, grow0 + g0);
            ptx::tma_load_2d(st + L::kZOff, &tmap_z, w_full(s), wt * (kTileN / PER), grow0 + g0);
          }
          ptx::mbar_arrive_expect_tx(full(s), L::kXBytes);
#pragma unroll
          for (int xb = 0; xb < SK / kSlabK; ++xb)
            ptx::tma_load_2d(st + xb * BT * 128, &tmap_x, full(s), kb * SK + xb * kSlabK, tr.row0);
        }
      }
      if (!ok) {  // let the copies already in flight land before the CTA releases its smem
        for (int j = it > NS ? it - NS : 0; j < it; ++j) {
          ptx::mbar_wait_drain(w_full(j % NS), (j / NS) & 1);
          ptx::mbar_wait_drain(full(j % NS), (j / NS) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      int it = 0, tcount = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++tcount) {
        const int b = ND == 2 ? (tcount & 1) : 0;
        const int use = ND == 2 ? (tcount >> 1) : tcount;   // earlier uses of this buffer
        if (!ptx::mbar_wait_sleep(d_empty(b), (use & 1) ^ 1, abort_flag)) break;
        ptx::tc_fence_after();
        for (int kb = 0; kb < nslab; ++kb, ++it) {
          const int s = it % NS;
          const uint32_t par = (it / NS) & 1;
          if (!ptx::mbar_wait_sleep(full(s), par, abort_flag) || !ptx::mbar_wait_sleep(a_full(s), par, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t xs = sbase + s * L::kStageBytes;
#pragma unroll
          for (int j = 0; j < SK / 16; ++j) {
            // K step j: activation box j / 4, 32-byte column (j % 4) of its swizzled rows
            ptx::mma_f16_ts(tmem + b * DCOL, tmem + A_COL + s * TCOLS_A + j * 8,
                            ptx::smem_desc_sw128(xs + (j >> 2) * BT * 128 + (j & 3) * 32), IDESC, (kb | j) != 0);
          }
          ptx::mma_commit(slab_free(s));  // frees the stage's shared memory and its TMEM A columns
        }
        if (ok) ptx::mma_commit(d_full(b));
      }
      // every MMA this thread issued has completed before TMEM is released (also on abort)
      ptx::mma_commit(fin_bar);
      ptx::mbar_wait_drain(fin_bar, 0);
    }
  } else if (warp >= kDequantWarp0 && warp < kDequantWarp0 + kDequantWarps) {
    // ---------------- dequant: lane = TMEM lane = output column. With DQ_ALT the two groups of
    // four warps take alternate stages and a warp converts both halves of its stage's K (one
    // ring wait and one TMEM-store wait per twice the work); otherwise warp group h converts
    // half h of every stage.
    const int q = warp & 3, grp = (warp - kDequantWarp0) >> 2;
    const int lrow = q * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
    int it = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      for (int kb = 0; kb < nslab; ++kb, ++it) {
        if (DQ_ALT && (it & 1) != grp) continue;
        const int s = it % NS;
        if (!ptx::mbar_wait_sleep(w_full(s), (it / NS) & 1, abort_flag)) goto done;
        const unsigned char* stp = smem + s * L::kStageBytes;
        if constexpr (FMT == kFmtQ4K) {
          // this lane's row: d | dmin | scales[12] | qs[128]; the stage is half hb of the block,
          // sub-blocks 4hb .. 4hb + 3 = low / high nibbles of qs chunks 2hb and 2hb + 1. Values
          // are the reference's fp32 d*sc*q - dmin*m rounded once to fp16, in the (j, j + 4)
          // pair order of the activation staging.
          const uint4 hd = *reinterpret_cast<const uint4*>(stp + L::kSOff + lrow * 16);
          const uint4* qrow = reinterpret_cast<const uint4*>(stp + L::kWOff + lrow * 64);
          const int sw = (lrow >> 1) & 3;   // 64-byte swizzle: 16-byte chunk i sits at i ^ sw
          const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xffffu)));
          const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
          const int hb = kb & 1;
          const uint32_t ta = lane_addr + A_COL + s * TCOLS_A;
#pragma unroll
          for (int c = 0; c < 2; ++c) {   // 32 TMEM columns per qs chunk, stored as soon as formed
            uint32_t v[32];
            const uint4 qa = qrow[(2 * c) ^ sw];
            const uint4 qb = qrow[(2 * c + 1) ^ sw];
            const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              uint32_t sc, mn;
              q4k_scale_min(hd.y, hd.z, hd.w, 4 * hb + 2 * c + u, sc, mn);
              const float dl = __fmul_rn(d, (float)sc), ml = __fmul_rn(dmin, (float)mn);
#pragma unroll
              for (int g = 0; g < 4; ++g) {
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                  // q as fp32 without a conversion instruction: 2^23 + q has q in its low
                  // mantissa bits, and subtracting 2^23 is exact
                  const float f0 = __int_as_float(0x4B000000u | ((qw[2 * g] >> (8 * p + 4 * u)) & 15u)) - 8388608.f;
                  const float f1 = __int_as_float(0x4B000000u | ((qw[2 * g + 1] >> (8 * p + 4 * u)) & 15u)) - 8388608.f;
                  v[u * 16 + 4 * g + p] = h2_as_u32(__floats2half2_rn(fmaf(dl, f0, -ml), fmaf(dl, f1, -ml)));
                }
              }
            }
            ptx::tmem_st32(ta + 32 * c, v);
          }
        } else {
        const uint32_t* wsm = reinterpret_cast<const uint32_t*>(stp + L::kWOff);
#pragma unroll
        for (int hh = 0; hh < (DQ_ALT ? 2 : 1); ++hh) {
          const int h = DQ_ALT ? hh : grp;
          const int gi = a.gb == 2 ? h : 0;   // scale/zero row of this half inside the stage
          uint32_t w[HROWS];
#pragma unroll
          for (int r = 0; r < HROWS; ++r) w[r] = wsm[(h * HROWS + r) * kTileN + lrow];
          const float scv = load_as_float(stp + L::kSOff, a.sc_dtype, gi * kTileN + lrow);
          const uint32_t zw = reinterpret_cast<const uint32_t*>(stp + L::kZOff)[gi * (kTileN / PER) + lrow / PER];
          const float zf = (float)((zw >> (BITS * (lrow % PER))) & MASK) + a.zoff;
          const uint32_t zlo = h2_as_u32(__float2half2_rn(1024.f + zf));
          const uint32_t zhi = h2_as_u32(__float2half2_rn(-(64.f + zf)));
          const __half2 s2 = __float2half2_rn(scv);
          uint32_t v[TCOLS_A / 2];   // this half's TMEM columns: SK / 4
#pragma unroll
          for (int r = 0; r < HROWS; ++r) {
            if constexpr (BITS == 4) {
              dq_int4(w[r], zlo, zhi, s2, &v[r * 4]);
            } else {
              dq_int8(w[r], zlo, s2, &v[r * 2]);
            }
          }
          const uint32_t ta = lane_addr + A_COL + s * TCOLS_A + h * (TCOLS_A / 2);
          if constexpr (TCOLS_A / 2 == 16) {
            ptx::tmem_st16(ta, v);
          } else {
#pragma unroll
            for (int c = 0; c < TCOLS_A / 2; c += 32)
              ptx::tmem_st32(ta + c, *reinterpret_cast<const uint32_t(*)[32]>(&v[c]));
          }
        }
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(a_full(s));
      }
    }
  } else if (warp >= kEpilogueWarp0) {
    // ---------------- epilogue: thread = TMEM lane = output column while draining TMEM (TMEM
    // columns = tokens). Each 32-token chunk goes through a per-warp [32 tokens][32 columns]
    // shared-memory transpose, after which a lane scales and stores 4 consecutive columns of one
    // token: 8 lanes write a 128-byte row segment, 8 wide stores per chunk instead of 32 narrow.
    const int q = warp & 3;
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
    float* stg = reinterpret_cast<float*>(smem + L::kEpiOff) + q * 32 * 32;
    const int r8 = lane >> 3, c4 = (lane & 7) * 4;   // store role: rows r8 + 4i, columns c4 .. c4 + 3
    const int osz = a.out_dtype == QL_F32 ? 4 : 2;
    const bool wide = (a.ldo & 3) == 0 && (reinterpret_cast<uintptr_t>(a.out) & (4 * osz - 1)) == 0;
    int tcount = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++tcount) {
      const int b = ND == 2 ? (tcount & 1) : 0;
      const int use = ND == 2 ? (tcount >> 1) : tcount;
      const int wt = tile % a.n_wtiles;
      const TileRows tr = tile_rows(a, tile / a.n_wtiles, BT);
      const int n4 = wt * kTileN + q * 32 + c4;   // N % 16 == 0: n4 < N covers all four columns
      float bias[4] = {0.f, 0.f, 0.f, 0.f};
      if (a.bias && n4 < a.N) {
#pragma unroll
        for (int i = 0; i < 4; ++i) bias[i] = a.bias[n4 + i];
      }
      int rexp[BT / 32];   // row exponent of token c * 32 + lane (broadcast with shuffles below)
#pragma unroll
      for (int c = 0; c < BT / 32; ++c) {
        const int tok = tr.row0 + c * 32 + lane;
        rexp[c] = tok < tr.row_end ? a.row_exp[tok] : 0;
      }
      if (!ptx::mbar_wait_sleep(d_full(b), use & 1, abort_flag)) goto done;
      ptx::tc_fence_after();
#pragma unroll
      for (int c = 0; c < BT / 32; ++c) {
        uint32_t v[32];
        ptx::tmem_ld32(lane_addr + b * DCOL + c * 32, v);
        ptx::tmem_wait_ld();
        if (c == BT / 32 - 1) {
          ptx::tc_fence_before();
          ptx::mbar_arrive(d_empty(b));  // accumulator drained into registers
        }
        __syncwarp();   // the previous chunk's reads of the transpose are done
#pragma unroll
        for (int j = 0; j < 32; ++j) stg[j * 32 + lane] = __uint_as_float(v[j]);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = 4 * i + r8;
          const int tok = tr.row0 + c * 32 + r;
          const float s = exp2i(__shfl_sync(0xffffffffu, rexp[c], r));
          if (n4 < a.N && tok < tr.row_end) {
            const float4 u = *reinterpret_cast<const float4*>(stg + r * 32 + c4);
            const float o[4] = {u.x * s + bias[0], u.y * s + bias[1], u.z * s + bias[2], u.w * s + bias[3]};
            const long idx = (long)tok * a.ldo + n4;
            if (wide && a.out_dtype == QL_F32) {
              *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + idx) = make_float4(o[0], o[1], o[2], o[3]);
            } else if (wide && a.out_dtype == QL_F16) {
              uint2 h;
              h.x = h2_as_u32(__floats2half2_rn(o[0], o[1]));
              h.y = h2_as_u32(__floats2half2_rn(o[2], o[3]));
              *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(a.out) + idx) = h;
            } else if (wide && a.out_dtype == QL_BF16) {
              const __nv_bfloat162 h0 = __floats2bfloat162_rn(o[0], o[1]), h1 = __floats2bfloat162_rn(o[2], o[3]);
              uint2 h;
              h.x = *reinterpret_cast<const uint32_t*>(&h0);
              h.y = *reinterpret_cast<const uint32_t*>(&h1);
              *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.out) + idx) = h;
            } else {
#pragma unroll
              for (int k = 0; k < 4; ++k) store_from_float(a.out, a.out_dtype, idx + k, o[k]);
            }
          }
        }
      }
    }
  }
done:
  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) atomicExch(&g_tc_status, 1);
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
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

bool encode(EncodeTiledFn enc, CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
            uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// n_experts: stacked weight matrices (grouped mode), 1 otherwise. FMT = kFmtQ4K: a.qw is the raw
// Q4_K tensor [N rows][K / 256 blocks of 144 bytes].
template <int BITS, int BT, int SK = kSlabK, bool DQ_ALT = false, int FMT = kFmtGptq>
int launch_gemm(const GemmArgs& a, const __half* x16, int n_experts, cudaStream_t st) {
  // ring depth: the TMEM A stages (NS * SK / 2 columns) fit beside the two BT-column
  // accumulators, the stages in shared memory beside the epilogue's transpose (even with
  // alternating dequant groups, at most 16)
  constexpr int kStage = SmemLayout<BITS, 1, BT, SK, FMT>::kStageBytes;
  constexpr int NS_T = (512 - 2 * BT) / (SK / 2);
  constexpr int NS_S = (227 * 1024 - 4 * 32 * 32 * 4 - 2048 - 1024) / kStage;
  constexpr int NS0 = NS_T < NS_S ? (NS_T < 16 ? NS_T : 16) : (NS_S < 16 ? NS_S : 16);
  constexpr int NS = DQ_ALT ? (NS0 & ~1) : NS0;
  constexpr int PER = 32 / BITS;
  using L = SmemLayout<BITS, NS, BT, SK, FMT>;
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    set_error("ql_gptq_matmul: cuTensorMapEncodeTiled is unavailable");
    return QL_ERR_CUDA;
  }
  const int G = a.K / a.gs;
  const int scb = a.sc_dtype == QL_F32 ? 4 : 2;
  const CUtensorMapDataType sdt = a.sc_dtype == QL_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                  : a.sc_dtype == QL_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tx, tw, ts, tz;
  bool ok = encode(enc, &tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x16, a.K, a.M, (uint64_t)a.K * 2, kSlabK, BT,
                   CU_TENSOR_MAP_SWIZZLE_128B);
  if (FMT == kFmtQ4K) {
    // two views of the rows: 64 quant bytes (one half super-block) and the 16-byte headers
    const uint64_t row_bytes = (uint64_t)(a.K / 256) * kQ4kBlockBytes;   // a multiple of 16
    ok = ok && encode(enc, &tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.qw, row_bytes, (uint64_t)a.N, row_bytes, 64,
                      kTileN, CU_TENSOR_MAP_SWIZZLE_64B) &&
         encode(enc, &ts, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.qw, row_bytes, (uint64_t)a.N, row_bytes, 16, kTileN,
                CU_TENSOR_MAP_SWIZZLE_NONE);
    tz = ts;   // unused by this format
  } else {
    ok = ok &&
         encode(enc, &tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.qw, a.N, (uint64_t)n_experts * (a.K / PER),
                (uint64_t)a.N * 4, kTileN, L::ROWS, CU_TENSOR_MAP_SWIZZLE_NONE) &&
         encode(enc, &ts, sdt, a.sc, a.N, (uint64_t)n_experts * G, (uint64_t)a.N * scb, kTileN, a.gb,
                CU_TENSOR_MAP_SWIZZLE_NONE) &&
         encode(enc, &tz, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.qz, a.N / PER, (uint64_t)n_experts * G,
                (uint64_t)(a.N / PER) * 4, kTileN / PER, a.gb, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (!ok) {
    set_error("ql_gptq_matmul: cuTensorMapEncodeTiled failed");
    return QL_ERR_CUDA;
  }
  auto kern = gptq_gemm_tc_kernel<BITS, NS, BT, SK, DQ_ALT, FMT>;
  static_assert(L::kBytes <= 227 * 1024, "shared memory per CTA");
  const int smem = L::kBytes;
  static int configured_dev = -1;
  static int sms = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                         "cudaFuncSetAttribute(gemm smem)");
    if (rc) return rc;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    configured_dev = dev;
  }
  const int ntiles = a.n_wtiles * a.n_ttiles;   // grouped mode: n_ttiles is the table's capacity
  const int grid = ntiles < sms ? ntiles : sms;
  kern<<<grid, kThreads, smem, st>>>(tx, tw, ts, tz, a);
  return cuda_status(cudaGetLastError(), "gptq_gemm_tc launch");
}

}  // namespace

size_t gptq_gemm_workspace(int M, int K) {
  return (((size_t)M * K * 2 + 255) & ~(size_t)255) + (size_t)M * 4 + 256;
}

// True when a call of this shape takes the tensor-core (large-M) path below.
bool gemm_path_taken(int M, int K, int gs) {
  static int min_m = -1;
  // measured: from 17 tokens on the tensor-core path beats the decode GEMV's 8-token slices
  // (M = 24 / 32 / 48 on 4096x11008: 24.7 / 24.8 / 25.8 us against 36.7 / 42.8 / 65.9); up to 16
  // tokens (the decode range) the GEMV keeps its per-group 23-bit activation staging
  if (min_m < 0) min_m = env_int("QL_GEMM_MIN_M", 17);
  return M >= min_m && K % kSlabK == 0 && (gs % 64 == 0 || gs == 32);
}

// Large-M path. *handled = false leaves the call to the GEMV path.
int gptq_gemm_sm100(const void* x, int x_dtype, long ldx, const int32_t* x_perm, const int32_t* qweight,
                    const int32_t* qzeros, const void* scales, int sc_dtype, const float* bias, void* out,
                    int out_dtype, long ldo, int M, int K, int N, int gs, int bits, float zoff, cudaStream_t st,
                    void* workspace, size_t ws_bytes, bool* handled) {
  *handled = false;
  if (!gemm_path_taken(M, K, gs)) return QL_OK;
  // TMA of the zero points: rows of N / per words must be whole 16-byte units, 16-byte aligned
  if (N % (4 * (32 / bits)) != 0 || (reinterpret_cast<uintptr_t>(qzeros) & 15)) return QL_OK;
  *handled = true;
  const size_t need = gptq_gemm_workspace(M, K);
  void* ws = workspace;
  bool owned = false;
  if (ws == nullptr || ws_bytes < need) {
    if (ws != nullptr) {
      set_error("ql_gptq_matmul: workspace of %zu bytes is smaller than the %zu needed", ws_bytes, need);
      return QL_ERR_ARG;
    }
    int rc = stream_alloc(&ws, need, st, "ql_gptq_matmul: workspace");
    if (rc) return rc;
    owned = true;
  }
  __half* x16 = reinterpret_cast<__half*>(ws);
  int* row_exp = reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + (((size_t)M * K * 2 + 255) & ~(size_t)255));
  int rc = launch_prep_x(bits, x, x_dtype, ldx, x_perm, nullptr, M, K, x16, row_exp, st);
  if (!rc) {
    GemmArgs a = {};
    a.qw = reinterpret_cast<const uint32_t*>(qweight);
    a.qz = reinterpret_cast<const uint32_t*>(qzeros);
    a.sc = scales; a.sc_dtype = sc_dtype; a.bias = bias; a.row_exp = row_exp;
    a.out = out; a.ldo = ldo; a.out_dtype = out_dtype;
    a.M = M; a.K = K; a.N = N; a.gs = gs; a.zoff = zoff;
    a.n_wtiles = (N + kTileN - 1) / kTileN;
    a.gb = gs == 32 ? 2 : 1;
    const bool half_tile = M <= 64 && K % 128 == 0 && gs % 128 == 0;   // one 64-token tile, deeper ring
    a.n_ttiles = half_tile ? 1 : (M + 127) / 128;
    if (half_tile)
      rc = bits == 4 ? launch_gemm<4, 64, 128, true>(a, x16, 1, st) : launch_gemm<8, 64, 128, true>(a, x16, 1, st);
    else if (K % 128 == 0 && gs % 128 == 0)   // 128-value stages (one scale row each), dequant groups alternating
      rc = bits == 4 ? launch_gemm<4, 128, 128, true>(a, x16, 1, st) : launch_gemm<8, 128, 128, true>(a, x16, 1, st);
    else
      rc = bits == 4 ? launch_gemm<4, 128>(a, x16, 1, st) : launch_gemm<8, 128>(a, x16, 1, st);
  }
  if (owned) {
    const int rc2 = cuda_status(cudaFreeAsync(ws, st), "cudaFreeAsync(workspace)");
    if (!rc) rc = rc2;
  }
  return rc;
}

// GGUF Q4_K GEMM (M >= kQ4kGemmMinM): the same pipeline with the Q4_K dequant role reading each
// row's super-blocks in place. Tiles of 32 / 64 / 128 tokens by M. *handled = false leaves the
// call to the decode kernels (N not a multiple of 16, M below the threshold).
int q4k_gemm_min_m() {
  static int min_m = -1;
  // below 16 tokens the decode GEMV stays, for its activation precision next to outlier channels
  // (this path stages x as fp16 with one exponent per row), although M = 8 / 12 measured
  // 33.7 / 34.0 us here against 35.2 / 53.5 through it
  if (min_m < 0) min_m = env_int("QL_Q4K_GEMM_MIN_M", 16);
  return min_m;
}

int q4k_gemm_sm100(const void* x, int x_dtype, long ldx, const uint8_t* raw, const float* bias, void* out,
                   int out_dtype, long ldo, int M, int K, int N, void* workspace, size_t ws_bytes, cudaStream_t st,
                   bool* handled) {
  *handled = false;
  if (M < q4k_gemm_min_m() || K % 256 != 0 || N % 16 != 0) return QL_OK;
  *handled = true;
  const size_t need = gptq_gemm_workspace(M, K);
  void* ws = workspace;
  bool owned = false;
  if (ws == nullptr || ws_bytes < need) {
    if (ws != nullptr) {
      set_error("ql_q4k_matmul: workspace of %zu bytes is smaller than the %zu needed", ws_bytes, need);
      return QL_ERR_ARG;
    }
    int rc = stream_alloc(&ws, need, st, "ql_q4k_matmul: workspace");
    if (rc) return rc;
    owned = true;
  }
  __half* x16 = reinterpret_cast<__half*>(ws);
  int* row_exp = reinterpret_cast<int*>(reinterpret_cast<char*>(ws) + (((size_t)M * K * 2 + 255) & ~(size_t)255));
  int rc = launch_prep_x(4, x, x_dtype, ldx, nullptr, nullptr, M, K, x16, row_exp, st);
  if (!rc) {
    GemmArgs a = {};
    a.qw = reinterpret_cast<const uint32_t*>(raw);
    a.bias = bias; a.row_exp = row_exp;
    a.out = out; a.ldo = ldo; a.out_dtype = out_dtype;
    a.M = M; a.K = K; a.N = N; a.gs = 256; a.zoff = 0.f; a.sc_dtype = QL_F16;
    a.n_wtiles = (N + kTileN - 1) / kTileN;
    a.gb = 1;
    const int bt = M <= 32 ? 32 : M <= 64 ? 64 : 128;
    a.n_ttiles = (M + bt - 1) / bt;
    rc = bt == 32 ? launch_gemm<4, 32, 128, true, kFmtQ4K>(a, x16, 1, st)
         : bt == 64 ? launch_gemm<4, 64, 128, true, kFmtQ4K>(a, x16, 1, st)
                    : launch_gemm<4, 128, 128, true, kFmtQ4K>(a, x16, 1, st);
  }
  if (owned) {
    const int rc2 = cuda_status(cudaFreeAsync(ws, st), "cudaFreeAsync(workspace)");
    if (!rc) rc = rc2;
  }
  return rc;
}

// Grouped (MoE) GEMM over P permuted rows: x rows gathered through row_map, experts' weights
// strided by *_estride elements, tiles from the device-built table (capacity max_tiles). With glu
// (== K) each x row is a fused [gate | up] row of 2K values, staged as their SwiGLU.
int gptq_gemm_grouped(const void* x, int x_dtype, long ldx, const int32_t* row_map, int P, const int32_t* qweight,
                      const int32_t* qzeros, const void* scales, int sc_dtype, long qw_estride, long qz_estride,
                      long sc_estride, const int32_t* offsets, const int32_t* tiles, const int32_t* n_tiles,
                      int max_tiles, int tile_rows_n, int n_experts, void* out, int out_dtype, long ldo, int K,
                      int N, int gs, int bits, float zoff, void* workspace, size_t ws_bytes, cudaStream_t st,
                      int glu) {
  if (K % kSlabK != 0 || (gs % 64 != 0 && gs != 32) || N % (4 * (32 / bits)) != 0 ||
      (reinterpret_cast<uintptr_t>(qzeros) & 15)) {
    set_error("grouped GEMM: K=%d must be a multiple of 64, gs=%d a multiple of 64 or 32, N=%d of 32 (int4) / 16 "
              "(int8), qzeros 16-byte aligned", K, gs, N);
    return QL_ERR_UNSUPPORTED;
  }
  if (tile_rows_n != 32 && tile_rows_n != 64 && tile_rows_n != kBT) {
    set_error("grouped GEMM: tile rows must be 32, 64 or %d (got %d)", kBT, tile_rows_n);
    return QL_ERR_ARG;
  }
  const size_t need = gptq_gemm_workspace(P, K);
  if (!workspace || ws_bytes < need) {
    set_error("grouped GEMM: workspace of %zu bytes needed", need);
    return QL_ERR_ARG;
  }
  __half* x16 = reinterpret_cast<__half*>(workspace);
  int* row_exp = reinterpret_cast<int*>(reinterpret_cast<char*>(workspace) + (((size_t)P * K * 2 + 255) & ~(size_t)255));
  if (P == 0) return QL_OK;
  int rc = launch_prep_x(bits, x, x_dtype, ldx, nullptr, row_map, P, K, x16, row_exp, st, glu);
  if (rc) return rc;
  GemmArgs a = {};
  a.qw = reinterpret_cast<const uint32_t*>(qweight);
  a.qz = reinterpret_cast<const uint32_t*>(qzeros);
  a.sc = scales; a.sc_dtype = sc_dtype; a.bias = nullptr; a.row_exp = row_exp;
  a.out = out; a.ldo = ldo; a.out_dtype = out_dtype;
  a.M = P; a.K = K; a.N = N; a.gs = gs; a.zoff = zoff;
  a.n_wtiles = (N + kTileN - 1) / kTileN;
  a.n_ttiles = max_tiles;
  a.tiles = tiles; a.n_tiles = n_tiles; a.offsets = offsets;
  a.qw_estride = qw_estride; a.qz_estride = qz_estride; a.sc_estride = sc_estride;
  a.gb = gs == 32 ? 2 : 1;
  if (K % 128 == 0 && gs % 128 == 0) {   // 128-value stages (one scale row each)
    switch (tile_rows_n) {
      case 32: return bits == 4 ? launch_gemm<4, 32, 128>(a, x16, n_experts, st) : launch_gemm<8, 32, 128>(a, x16, n_experts, st);
      case 64: return bits == 4 ? launch_gemm<4, 64, 128>(a, x16, n_experts, st) : launch_gemm<8, 64, 128>(a, x16, n_experts, st);
      default:
        return bits == 4 ? launch_gemm<4, 128, 128, true>(a, x16, n_experts, st)
                         : launch_gemm<8, 128, 128, true>(a, x16, n_experts, st);
    }
  }
  switch (tile_rows_n) {
    case 32: return bits == 4 ? launch_gemm<4, 32>(a, x16, n_experts, st) : launch_gemm<8, 32>(a, x16, n_experts, st);
    case 64: return bits == 4 ? launch_gemm<4, 64>(a, x16, n_experts, st) : launch_gemm<8, 64>(a, x16, n_experts, st);
    default: return bits == 4 ? launch_gemm<4, 128>(a, x16, n_experts, st) : launch_gemm<8, 128>(a, x16, n_experts, st);
  }
}

int take_tc_status() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(int));
  const int zero = 0;
  cudaMemcpyToSymbol(g_tc_status, &zero, sizeof(int));
  return v;
}

}  // namespace ql

namespace ql {
size_t gemv_stage_workspace(int M, int K, int kgs);
}

// The larger of the two paths' needs: the tensor-core path's fp16 staging, and the decode path's
// staged activations for up to 16 tokens a launch (counted for 32-value groups, the most sums).
extern "C" size_t ql_gptq_matmul_workspace(int M, int K) {
  if (M <= 0 || K <= 0) return 0;
  const size_t gemm = ql::gptq_gemm_workspace(M, K);
  const size_t gemv = ql::gemv_stage_workspace(M < 16 ? M : 16, K, 32);
  return gemm > gemv ? gemm : gemv;
}

namespace ql {
int take_tma_gemv_status();
int take_q4k_tma_status();
}

extern "C" int ql_device_status(void) {
  const cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return ql::cuda_status(e, "ql_device_status");
  const int gemm = ql::take_tc_status();
  const int gemv = ql::take_tma_gemv_status() | ql::take_q4k_tma_status();
  if (gemm || gemv) {
    ql::set_error("a tensor-core kernel gave up on a bounded wait");
    return QL_ERR_TIMEOUT;
  }
  return QL_OK;
}

// ---------------------------------------------------------------------------------------
// allocation-free entry point
// ---------------------------------------------------------------------------------------
namespace ql {
// Some callers cannot allocate device memory at call time: hosts that hand out every byte of
// device memory through their own allocator or a fixed budget (inference servers, plugin
// sandboxes, language bindings with no handle on a CUDA allocator) and code that must not
// allocate while it runs under a latency budget. For them the only scratch this library needs
// -- the large-M path's fp16 activation staging plus one int per row -- lives in the fixed
// array below, which every GPU that loads the library holds until the process exits.
namespace {

constexpr size_t kNoAllocScratchBytes = 24ull << 20;  // 24 MiB: M * K up to ~12.5 M activations
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch array in the current device's context. The host-side symbol is
// only a stand-in; a kernel must be given this address. It is looked up on every call (the
// lookup allocates nothing), so a context torn down and created again never leaves a stale one.
int noalloc_scratch(void** out) {
  void* p = nullptr;
  const int rc = cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch), "ql_gptq_matmul_noalloc: cudaGetSymbolAddress");
  if (rc) return rc;
  *out = p;
  return QL_OK;
}

}  // namespace

int gptq_matmul_impl(const void* x, int x_dtype, long ldx, const int32_t* x_perm, const int32_t* qweight,
                     const int32_t* qzeros, const void* scales, int scales_dtype, const float* bias, void* out,
                     int out_dtype, long ldo, int M, int K, int N, int gs, int bits, float zero_offset,
                     void* stream, void* workspace, size_t ws_bytes);
}  // namespace ql

extern "C" size_t ql_gptq_matmul_noalloc_max_scratch(void) { return ql::kNoAllocScratchBytes; }

extern "C" int ql_gptq_matmul_noalloc(const void* x, int x_dtype, long ldx, const int32_t* x_perm,
                                      const int32_t* qweight, const int32_t* qzeros, const void* scales,
                                      int scales_dtype, const float* bias, void* out, int out_dtype, long ldo,
                                      int M, int K, int N, int gs, int bits, float zero_offset, void* stream) {
  void* ws = nullptr;
  size_t ws_bytes = 0;
  const bool gemm = M > 0 && K > 0 && gs > 0 && ql::gemm_path_taken(M, K, gs);
  if (gemm || (M > 4 && K > 0 && gs > 0)) {   // tensor-core path, or staged decode activations
    const size_t need = gemm ? ql::gptq_gemm_workspace(M, K) : ql::gemv_stage_workspace(M < 16 ? M : 16, K, 32);
    if (need > ql::kNoAllocScratchBytes) {
      ql::set_error("ql_gptq_matmul_noalloc: M=%d x K=%d needs %zu bytes of scratch; this entry point has %zu "
                    "(use ql_gptq_matmul_ws with a workspace, or split M)",
                    M, K, need, ql::kNoAllocScratchBytes);
      return QL_ERR_UNSUPPORTED;
    }
    const int rc = ql::noalloc_scratch(&ws);
    if (rc) return rc;
    ws_bytes = ql::kNoAllocScratchBytes;
  }
  // no path below may fall back to the stream-ordered allocator: it fails instead
  const ql::AllocGuard no_alloc;
  return ql::gptq_matmul_impl(x, x_dtype, ldx, x_perm, qweight, qzeros, scales, scales_dtype, bias, out, out_dtype,
                              ldo, M, K, N, gs, bits, zero_offset, stream, ws, ws_bytes);
}
