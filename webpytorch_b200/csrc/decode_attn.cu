// One decode position of grouped-query attention with rotary embedding and a KV cache, the step
// that sits between the QKV and O projections of a decode layer.
//
// Reference semantics (webtorch/lm_engine.py:66-74 `_rope` / `_rot`, 89-101 `_block`;
// webtorch/llm.py:1591-1612 `_decode_fwd`): q and k are rotated with rotate-half,
//   r[i] = x[i] cos_i - x[i + HD/2] sin_i,  r[i + HD/2] = x[i + HD/2] cos_i + x[i] sin_i,
// the position's k and v go into the cache, and each query head h attends over positions
// 0 .. pos of its key/value head h / (NH / NKV): softmax(q . K^T * scale) . V, in fp32.
//
// The position is read from device memory (pos[0]) so a captured CUDA graph replays the same
// launch for every token; the grid covers the whole cache and CTAs past the position leave at
// once. Work is split over positions (split-softmax): CTA (h, j) takes positions 64 j .. 64 j +
// 63, writes its running maximum, sum of exponentials and unnormalised output to the workspace,
// and the last CTA of head h to finish (a per-head counter that it resets to zero) combines them.
// A CTA uses its own rotated k and v for position pos (no read-after-write through the cache
// inside the launch); the CTA of the first head of each group that holds pos writes them to the
// cache for later steps.
#include "ql_common.cuh"

namespace ql {
namespace {

constexpr int kThreads = 128;
constexpr int kChunk = 64;    // positions per CTA

__global__ void __launch_bounds__(kThreads) decode_attention_kernel(
    const float* __restrict__ qkv, int NH, int NKV, int HD, const float* __restrict__ rope_cos,
    const float* __restrict__ rope_sin, const int32_t* __restrict__ pos_ptr, float* __restrict__ kcache,
    float* __restrict__ vcache, int lmax, float scale, float* __restrict__ out, float* __restrict__ part,
    unsigned int* __restrict__ counters) {
  extern __shared__ float sm[];
  float* qr = sm;             // [HD] rotated query
  float* kr = qr + HD;        // [HD] rotated key of position pos
  float* vr = kr + HD;        // [HD] value of position pos
  float* sc = vr + HD;        // [max(kChunk, splits)] scores, then exponentials, then chunk weights
  __shared__ float red[kThreads / 32];
  __shared__ bool last;
  const int h = blockIdx.x, j = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int group = NH / NKV, g = h / group;
  // launched as a programmatic dependent: q, k, v and the position are the previous kernel's
  // output (every CTA waits before anything else, so this grid never completes ahead of it);
  // the next kernel (the O projection) may then start streaming its weights
  pdl_wait();
  pdl_trigger();
  const int pos = *pos_ptr;
  const int half = HD / 2;
  if (pos < 0 || pos >= lmax) {   // a position outside the cache: NaN output, nothing written
    if (j == 0)
      for (int d = tid; d < HD; d += kThreads) out[(long)h * HD + d] = __int_as_float(0x7fc00000);
    return;
  }
  const int p0 = j * kChunk;
  if (p0 > pos) return;           // this CTA's positions are all past the current one
  const int np = min(kChunk, pos + 1 - p0);
  const int nsplit = pos / kChunk + 1;
  const float* q = qkv + (long)h * HD;
  const float* k = qkv + (long)NH * HD + (long)g * HD;
  const float* v = qkv + (long)(NH + NKV) * HD + (long)g * HD;
  const float* cs = rope_cos + (long)pos * half;
  const float* sn = rope_sin + (long)pos * half;
  const bool has_pos = pos < p0 + kChunk;
  for (int i = tid; i < half; i += kThreads) {
    const float c = cs[i], s = sn[i];
    const float q1 = q[i], q2 = q[i + half];
    qr[i] = q1 * c - q2 * s;
    qr[i + half] = q2 * c + q1 * s;
    if (has_pos) {
      const float k1 = k[i], k2 = k[i + half];
      kr[i] = k1 * c - k2 * s;
      kr[i + half] = k2 * c + k1 * s;
    }
  }
  if (has_pos)
    for (int i = tid; i < HD; i += kThreads) vr[i] = v[i];
  __syncthreads();
  const float* kc = kcache + (long)g * lmax * HD;
  const float* vc = vcache + (long)g * lmax * HD;
  if (has_pos && h % group == 0) {
    for (int i = tid; i < HD; i += kThreads) {
      kcache[(long)g * lmax * HD + (long)pos * HD + i] = kr[i];
      vcache[(long)g * lmax * HD + (long)pos * HD + i] = vr[i];
    }
  }
  // scores: each warp takes 8 positions at a time (their key rows loaded together, 16 bytes a
  // lane), lanes over the head dimension
  constexpr int kPW = 8;
  for (int r0 = warp * kPW; r0 < np; r0 += (kThreads / 32) * kPW) {
    float s[kPW];
#pragma unroll
    for (int u = 0; u < kPW; ++u) {
      s[u] = 0.f;
      const int r = r0 + u;
      if (r < np) {
        const int p = p0 + r;
        const float* kp = p == pos ? kr : kc + (long)p * HD;
        for (int i = 4 * lane; i < HD; i += 128) {
          const float4 kk = *reinterpret_cast<const float4*>(kp + i);
          const float4 qq = *reinterpret_cast<const float4*>(qr + i);
          s[u] = fmaf(qq.x, kk.x, fmaf(qq.y, kk.y, fmaf(qq.z, kk.z, fmaf(qq.w, kk.w, s[u]))));
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < kPW; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], o);
    if (lane == 0)
#pragma unroll
      for (int u = 0; u < kPW; ++u)
        if (r0 + u < np) sc[r0 + u] = s[u] * scale;
  }
  __syncthreads();
  float mx = tid < np ? sc[tid] : -3.4e38f;
  if (kThreads < kChunk && tid + kThreads < np) mx = fmaxf(mx, sc[tid + kThreads]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < kThreads / 32; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  float sum = 0.f;
  if (tid < np) {
    const float e = expf(sc[tid] - mx);
    sc[tid] = e;
    sum = e;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  sum = 0.f;
  for (int w = 0; w < kThreads / 32; ++w) sum += red[w];
  // unnormalised partial output of this chunk: sum_p e_p V[p][d]
  float* pp = part + ((long)h * gridDim.y + j) * (HD + 2);
  for (int d = tid; d < HD; d += kThreads) {
    // 16 value rows in flight per thread (the loop is bound by load latency, not arithmetic)
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int r = 0;
    const int nc = np - (has_pos ? 1 : 0);   // positions read from the cache
    for (; r + 16 <= nc; r += 16) {
      float vv[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) vv[u] = vc[(long)(p0 + r + u) * HD + d];
#pragma unroll
      for (int u = 0; u < 16; ++u) acc[u & 3] = fmaf(sc[r + u], vv[u], acc[u & 3]);
    }
    for (; r < nc; ++r) acc[0] = fmaf(sc[r], vc[(long)(p0 + r) * HD + d], acc[0]);
    if (has_pos) acc[1] = fmaf(sc[np - 1], vr[d], acc[1]);
    pp[d] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  }
  if (tid == 0) {
    pp[HD] = mx;
    pp[HD + 1] = sum;
  }
  // the last chunk of head h to finish combines the chunks
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(&counters[h], 1u) == (unsigned)nsplit - 1u;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float* ph = part + (long)h * gridDim.y * (HD + 2);
  // other CTAs' partials: read past L1 (it is not coherent with their writes). The chunks'
  // weights exp(m_s - M) / L go to shared memory (sc, free again), one thread per chunk.
  float ms = -3.4e38f, ls = 0.f;
  if (tid < nsplit) {
    ms = __ldcg(ph + (long)tid * (HD + 2) + HD);
    ls = __ldcg(ph + (long)tid * (HD + 2) + HD + 1);
  }
  float M = ms;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  __syncthreads();
  if (lane == 0) red[warp] = M;
  __syncthreads();
  M = red[0];
  for (int w = 1; w < kThreads / 32; ++w) M = fmaxf(M, red[w]);
  const float e = tid < nsplit ? expf(ms - M) : 0.f;
  float L = e * ls;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  __syncthreads();
  if (lane == 0) red[warp] = L;
  if (tid < nsplit) sc[tid] = e;
  __syncthreads();
  L = 0.f;
  for (int w = 0; w < kThreads / 32; ++w) L += red[w];
  const float inv = 1.0f / L;
  for (int d = tid; d < HD; d += kThreads) {
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    int s = 0;
    for (; s + 8 <= nsplit; s += 8) {
      float pv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) pv[u] = __ldcg(ph + (long)(s + u) * (HD + 2) + d);
#pragma unroll
      for (int u = 0; u < 8; ++u) o[u & 3] = fmaf(pv[u], sc[s + u], o[u & 3]);
    }
    for (; s < nsplit; ++s) o[0] = fmaf(__ldcg(ph + (long)s * (HD + 2) + d), sc[s], o[0]);
    out[(long)h * HD + d] = ((o[0] + o[1]) + (o[2] + o[3])) * inv;
  }
  if (tid == 0) counters[h] = 0u;   // ready for the next launch
}

}  // namespace
}  // namespace ql

using namespace ql;

extern "C" size_t ql_decode_attention_workspace(int NH, int HD, int lmax) {
  if (NH <= 0 || HD <= 0 || lmax <= 0) return 0;
  const size_t nsplit = (size_t)(lmax + kChunk - 1) / kChunk;
  return (((size_t)NH * nsplit * (HD + 2) * sizeof(float) + 255) & ~(size_t)255) + (size_t)NH * sizeof(unsigned int);
}

extern "C" int ql_decode_attention(const float* qkv, int NH, int NKV, int HD, const float* rope_cos,
                                   const float* rope_sin, const int32_t* pos, float* kcache, float* vcache, int lmax,
                                   float scale, float* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!qkv || !rope_cos || !rope_sin || !pos || !kcache || !vcache || !out || !workspace || NH <= 0 || NKV <= 0 ||
      NH % NKV || HD <= 0 || HD % 8 || HD > 1024 || lmax <= 0 || (reinterpret_cast<uintptr_t>(kcache) & 15)) {
    set_error("ql_decode_attention: bad arguments (NH=%d NKV=%d HD=%d lmax=%d; HD a multiple of 8, caches 16-byte "
              "aligned)", NH, NKV, HD, lmax);
    return QL_ERR_ARG;
  }
  const size_t need = ql_decode_attention_workspace(NH, HD, lmax);
  if (workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255)) {
    set_error("ql_decode_attention: workspace of %zu bytes (256-byte aligned, counters zeroed once) needed", need);
    return QL_ERR_ARG;
  }
  const int nsplit = (lmax + kChunk - 1) / kChunk;
  float* part = reinterpret_cast<float*>(workspace);
  unsigned int* counters = reinterpret_cast<unsigned int*>(reinterpret_cast<char*>(workspace) + need -
                                                           (size_t)NH * sizeof(unsigned int));
  const size_t smem = (size_t)(3 * HD + (nsplit > kChunk ? nsplit : kChunk)) * sizeof(float);
  if (nsplit > kThreads) {
    set_error("ql_decode_attention: lmax=%d is above %d positions", lmax, kThreads * kChunk);
    return QL_ERR_UNSUPPORTED;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(NH, nsplit);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  if (launch_flags() & QL_LAUNCH_PDL) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cuda_status(cudaLaunchKernelEx(&cfg, decode_attention_kernel, qkv, NH, NKV, HD, rope_cos, rope_sin, pos,
                                        kcache, vcache, lmax, scale, out, part, counters),
                     "ql_decode_attention launch");
}
