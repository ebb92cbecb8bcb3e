// Attention for decoding: a few query rows per sequence (Tq <= 16 / group) against a KV cache of Tk
// keys, bottom-right aligned (query row t sits at position Tk - Tq + t). Memory-bound: every key
// and value row is read once.
//
// Split-KV ("flash decoding"): kernel 1 runs one CTA per (256-key chunk, KV head, batch row). Its
// 256 threads own one key each for the scores (the G * Tq query rows that share the KV head sit in
// shared memory as fp32), each warp then reduces two rows' scores to a chunk max and sum, and the
// P @ V product is taken with one head dimension per thread, so every value row is one coalesced
// 256-byte read. The chunk's partial (max, sum, unnormalized output) goes to an fp32 workspace;
// kernel 2 merges the chunks of each row with the usual log-sum-exp rescaling and writes bf16.
// Reference: the KV-cache branch of mint/nn/flashattn.py:171-216 (flash_attn_with_kvcache / SDPA).
#include <cmath>

#include "common.cuh"
#include "host_common.h"

namespace mint {
namespace dec {

constexpr int kD = 128;
constexpr int kChunk = 256;   // keys per CTA (one per thread)
constexpr int kMaxRows = 16;  // query rows per KV head (G * Tq)
constexpr int kThreads = 256;

struct Params {
  const __nv_bfloat16* q;  // [B, Tq, Hq, D] contiguous
  const __nv_bfloat16* k;  // [B, Tk, Hkv, D] rows contiguous, batch stride kv_bstride
  const __nv_bfloat16* v;
  __nv_bfloat16* o;        // [B, Tq, Hq, D]
  float* ws;               // [B, Hkv, nsplit, R, D + 2] (output partial, max, sum)
  long long kv_bstride;    // elements between batch rows of k / v
  int B, Tq, Tk, Hq, Hkv, R, nsplit, causal, window;
  float scale_log2;
};

__global__ void __launch_bounds__(kThreads) decode_partial_kernel(Params p) {
  __shared__ float qs[kMaxRows][kD];
  __shared__ float sc[kMaxRows][kChunk];
  __shared__ float mrow[kMaxRows], lrow[kMaxRows];
  const int s = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = p.Hq / p.Hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // query rows r = t * G + g (query position t, head hk * G + g)
  for (int i = tid; i < p.R * kD; i += kThreads) {
    const int r = i / kD, d = i % kD;
    const int t = r / G, g = r % G;
    qs[r][d] = __bfloat162float(p.q[((static_cast<long long>(b) * p.Tq + t) * p.Hq + hk * G + g) * kD + d]);
  }
  __syncthreads();
  // scores: thread = key
  const int j = s * kChunk + tid;
  float acc[kMaxRows];
#pragma unroll
  for (int r = 0; r < kMaxRows; ++r) acc[r] = 0.f;
  if (j < p.Tk) {
    const uint4* krow = reinterpret_cast<const uint4*>(p.k + b * p.kv_bstride + (static_cast<long long>(j) * p.Hkv + hk) * kD);
#pragma unroll 4
    for (int c = 0; c < kD / 8; ++c) {
      const uint4 u = krow[c];
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
      float kf[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h2[e]);
        kf[2 * e] = f.x;
        kf[2 * e + 1] = f.y;
      }
#pragma unroll
      for (int r = 0; r < kMaxRows; ++r) {
        if (r < p.R) {
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[r] = fmaf(qs[r][c * 8 + e], kf[e], acc[r]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kMaxRows; ++r) {
    if (r >= p.R) break;
    const int t = r / G;
    const int pos = p.Tk - p.Tq + t;  // this query row's position
    bool keep = j < p.Tk;
    if (p.causal) keep = keep && j <= pos;
    if (p.window >= 0) keep = keep && pos - j <= p.window;
    sc[r][tid] = keep ? acc[r] : -INFINITY;
  }
  __syncthreads();
  // per row: chunk max and sum of exp2((s - m) * scale_log2); warp w takes rows w and w + 8
  for (int r = warp; r < p.R; r += kThreads / 32) {
    float m = -INFINITY;
    for (int c = lane; c < kChunk; c += 32) m = fmaxf(m, sc[r][c]);
    m = warp_max(m);
    float l = 0.f;
    for (int c = lane; c < kChunk; c += 32) {
      const float e = (m == -INFINITY) ? 0.f : exp2f((sc[r][c] - m) * p.scale_log2);
      sc[r][c] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      mrow[r] = m;
      lrow[r] = l;
    }
  }
  __syncthreads();
  // P @ V: thread = (head dimension d, row parity); value rows are read coalesced
  const int d = tid & (kD - 1);
  const int par = tid >> 7;
  float o[kMaxRows / 2];
#pragma unroll
  for (int i = 0; i < kMaxRows / 2; ++i) o[i] = 0.f;
  const int jend = min(kChunk, p.Tk - s * kChunk);
  const __nv_bfloat16* vcol = p.v + b * p.kv_bstride + (static_cast<long long>(s) * kChunk * p.Hkv + hk) * kD + d;
  for (int c = 0; c < jend; ++c) {
    const float vv = __bfloat162float(vcol[static_cast<long long>(c) * p.Hkv * kD]);
#pragma unroll
    for (int i = 0; i < kMaxRows / 2; ++i) {
      const int r = 2 * i + par;
      if (r < p.R) o[i] = fmaf(sc[r][c], vv, o[i]);
    }
  }
  float* w = p.ws + ((static_cast<long long>(b) * p.Hkv + hk) * p.nsplit + s) * p.R * (kD + 2);
#pragma unroll
  for (int i = 0; i < kMaxRows / 2; ++i) {
    const int r = 2 * i + par;
    if (r < p.R) w[r * (kD + 2) + d] = o[i];
  }
  if (tid < p.R) {
    w[tid * (kD + 2) + kD] = mrow[tid];
    w[tid * (kD + 2) + kD + 1] = lrow[tid];
  }
}

// one CTA per (row, KV head, batch row), one thread per head dimension
__global__ void __launch_bounds__(kD) decode_combine_kernel(Params p) {
  const int r = blockIdx.x, hk = blockIdx.y, b = blockIdx.z, d = threadIdx.x;
  const int G = p.Hq / p.Hkv;
  const float* w = p.ws + (static_cast<long long>(b) * p.Hkv + hk) * p.nsplit * p.R * (kD + 2);
  float M = -INFINITY;
  for (int s = 0; s < p.nsplit; ++s) M = fmaxf(M, w[(s * p.R + r) * (kD + 2) + kD]);
  float L = 0.f, acc = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < p.nsplit; ++s) {
      const float* ws = w + (s * p.R + r) * (kD + 2);
      const float m = ws[kD];
      if (m == -INFINITY) continue;
      const float f = exp2f((m - M) * p.scale_log2);
      L = fmaf(ws[kD + 1], f, L);
      acc = fmaf(ws[d], f, acc);
    }
  }
  const int t = r / G, g = r % G;
  p.o[((static_cast<long long>(b) * p.Tq + t) * p.Hq + hk * G + g) * kD + d] =
      __float2bfloat16_rn(L > 0.f ? acc / L : 0.f);
}

}  // namespace dec

// o [B, Tq, Hq, D] = softmax(q k^T * scale) v over a KV cache prefix (k, v: [B, Tk, Hkv, D] with
// contiguous rows; the batch stride may be the cache's), causal bottom-right, optional window.
at::Tensor decode_attention(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, bool causal,
                            int64_t window, double scale) {
  check_contig(q, "q");
  check_cuda(k, "k");
  check_cuda(v, "v");
  MINT_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
             "decode attention expects bf16");
  MINT_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4 && q.size(3) == dec::kD && k.size(3) == dec::kD,
             "decode attention expects [B, T, H, 128]");
  const int B = static_cast<int>(q.size(0)), Tq = static_cast<int>(q.size(1)), Hq = static_cast<int>(q.size(2));
  const int Tk = static_cast<int>(k.size(1)), Hkv = static_cast<int>(k.size(2));
  MINT_CHECK(k.sizes() == v.sizes() && k.size(0) == B && Hq % Hkv == 0 && Tq <= Tk, "decode attention shapes");
  MINT_CHECK(k.stride(3) == 1 && k.stride(2) == dec::kD && k.stride(1) == Hkv * dec::kD && v.strides() == k.strides(),
             "k / v rows must be contiguous [.., Hkv, 128] with equal strides");
  const int R = (Hq / Hkv) * Tq;
  MINT_CHECK(R <= dec::kMaxRows, "decode attention takes at most 16 query rows per KV head");
  auto o = at::empty_like(q);
  if (B == 0 || Tq == 0) return o;
  const int nsplit = (Tk + dec::kChunk - 1) / dec::kChunk;
  auto ws = at::empty({static_cast<int64_t>(B) * Hkv * nsplit * R * (dec::kD + 2)}, q.options().dtype(at::kFloat));
  c10::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  dec::Params p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  p.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.ws = ws.data_ptr<float>();
  p.kv_bstride = k.stride(0);
  p.B = B;
  p.Tq = Tq;
  p.Tk = Tk;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.R = R;
  p.nsplit = nsplit;
  p.causal = causal ? 1 : 0;
  p.window = static_cast<int>(window);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  dec::decode_partial_kernel<<<dim3(nsplit, Hkv, B), dec::kThreads, 0, stream>>>(p);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  dec::decode_combine_kernel<<<dim3(R, Hkv, B), dec::kD, 0, stream>>>(p);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return o;
}

}  // namespace mint
