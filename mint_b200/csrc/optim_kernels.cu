// Optimizer kernels: NorMuon (reference: mint/optim/muon_adamw.py:94-149, 187-252) around the
// Polar-Express GEMM chain, the global gradient norm with the clip coefficient kept on the device,
// and the per-step refresh of the bf16 compute copies of the fp32 master weights.
//
// NorMuon on a stack of n equally shaped matrices (rows R, columns C):
//   prep   m <- lerp(m, s g, 1 - mu);  g' = lerp(s g, m, mu)  (Nesterov; s = clip coefficient), g' is
//          written over the gradient and ||g'||_F^2 accumulated per matrix
//   cast   X0 = bf16(g' / (1.01 ||g'||_F + 1e-6))                      -> Polar-Express GEMM chain
//   stats  per row (R >= C) or per column (R < C) sum of X^2
//   scale  v = mean of X^2 along the reduced dimension; v2 <- lerp(v2, v, 1 - beta2);
//          s_j = rsqrt(max(v2_j, 1e-10)); ratio = ||X||_F / ||X s||_F; writes s_j * ratio
//   apply  g = X s_j ratio; p <- p - lr g - lr wd p [g p >= 0]   (cautious weight decay)
// The matrices' gradients and parameters are addressed through device pointer tables (they are
// views into the gradient engine's buckets), so nothing is stacked or copied.
//
// Every update kernel (prep, scale, apply) returns without writing when the device status word is
// non-zero (a kernel of this step reported a timed-out wait): the step then changes no state.
#include "common.cuh"
#include "host_common.h"

namespace mint {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read by a previous call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  v = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
  if (warp == 0) v = warp_sum(v);
  return v;  // valid in thread 0
}

// grid (chunks, n): blockIdx.y = matrix. 4 elements per thread step (per % 4 == 0, 16-byte aligned).
__global__ void normuon_prep_kernel(const long long* __restrict__ gptrs, float* __restrict__ mb,
                                    float* __restrict__ sumsq, long long per, float mu,
                                    const float* __restrict__ gscale, const uint32_t* __restrict__ status) {
  __shared__ float red[32];
  if (status_failed(status)) return;
  const int i = blockIdx.y;
  float4* g4 = reinterpret_cast<float4*>(gptrs[i]);
  float4* m4 = reinterpret_cast<float4*>(mb + static_cast<long long>(i) * per);
  const float s = gscale != nullptr ? *gscale : 1.f;
  const long long n4 = per >> 2;
  float acc = 0.f;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n4;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 g = g4[e], m = m4[e];
    float* ga = &g.x;
    float* ma = &m.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gv = ga[k] * s;
      ma[k] = ma[k] + (1.f - mu) * (gv - ma[k]);
      ga[k] = gv + mu * (ma[k] - gv);
      acc = fmaf(ga[k], ga[k], acc);
    }
    g4[e] = g;
    m4[e] = m;
  }
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) atomicAdd(sumsq + i, acc);
}

// X0 = bf16(g' / (1.01 ||g'|| + 1e-6)); 8 elements per thread step (per % 8 == 0)
__global__ void normuon_cast_kernel(const long long* __restrict__ gptrs, const float* __restrict__ sumsq,
                                    __nv_bfloat16* __restrict__ X, long long per) {
  const int i = blockIdx.y;
  const float4* g4 = reinterpret_cast<const float4*>(gptrs[i]);
  uint4* x8 = reinterpret_cast<uint4*>(X + static_cast<long long>(i) * per);
  const float inv = 1.f / (1.01f * sqrtf(sumsq[i]) + 1e-6f);
  const long long n8 = per >> 3;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n8;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 a = g4[2 * e], b = g4[2 * e + 1];
    uint4 o;
    o.x = pack_bf16x2(a.x * inv, a.y * inv);
    o.y = pack_bf16x2(a.z * inv, a.w * inv);
    o.z = pack_bf16x2(b.x * inv, b.y * inv);
    o.w = pack_bf16x2(b.z * inv, b.w * inv);
    x8[e] = o;
  }
}

__device__ __forceinline__ float sq_bf16x8(const uint4 v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __bfloat1622float2(h[k]);
    acc = fmaf(f.x, f.x, acc);
    acc = fmaf(f.y, f.y, acc);
  }
  return acc;
}

// Row sums of squares (R >= C): one warp per row, C % 8 == 0. out[i * R + r]. grid (ceil(R / 8), n).
__global__ void normuon_rowstats_kernel(const __nv_bfloat16* __restrict__ X, float* __restrict__ out, int R, int C) {
  const int i = blockIdx.y;
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= R) return;
  const uint4* row = reinterpret_cast<const uint4*>(X + (static_cast<long long>(i) * R + r) * C);
  float acc = 0.f;
  for (int c = lane; c < (C >> 3); c += 32) acc += sq_bf16x8(row[c]);
  acc = warp_sum(acc);
  if (lane == 0) out[static_cast<long long>(i) * R + r] = acc;
}

// Column sums of squares (R < C): thread = two adjacent columns, blockIdx.z = one of S row slices.
// out[(s * n + i) * C + c]. grid (ceil(C / 512), n, S), 256 threads.
__global__ void normuon_colstats_kernel(const __nv_bfloat16* __restrict__ X, float* __restrict__ out, int R, int C,
                                        int n) {
  const int i = blockIdx.y;
  const int s = blockIdx.z, S = gridDim.z;
  const int c = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (c >= C) return;
  const int r0 = static_cast<int>(static_cast<long long>(R) * s / S);
  const int r1 = static_cast<int>(static_cast<long long>(R) * (s + 1) / S);
  const __nv_bfloat16* base = X + static_cast<long long>(i) * R * C + c;
  float a0 = 0.f, a1 = 0.f;
  for (int r = r0; r < r1; ++r) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(base + static_cast<long long>(r) * C));
    a0 = fmaf(f.x, f.x, a0);
    a1 = fmaf(f.y, f.y, a1);
  }
  float* o = out + (static_cast<long long>(s) * n + i) * C + c;
  o[0] = a0;
  o[1] = a1;
}

// One block per matrix: combine the S partial sums of the J statistics, update the second moment
// and write scale[i][j] = rsqrt(max(v2_j, 1e-10)) * ||X|| / ||X s||.
__global__ void normuon_scale_kernel(const float* __restrict__ partial, float* __restrict__ v2,
                                     float* __restrict__ scale, int n, int J, int S, float red, float beta2,
                                     const uint32_t* __restrict__ status) {
  __shared__ float sred[32];
  __shared__ float ratio_s;
  if (status_failed(status)) return;
  const int i = blockIdx.x;
  float nrm = 0.f, nrm_new = 0.f;
  for (int j = threadIdx.x; j < J; j += blockDim.x) {
    float sum = 0.f;
    for (int s = 0; s < S; ++s) sum += partial[(static_cast<long long>(s) * n + i) * J + j];
    const float vmean = sum / red;
    float* v = v2 + static_cast<long long>(i) * J + j;
    const float nv = *v + (1.f - beta2) * (vmean - *v);
    *v = nv;
    const float st = rsqrtf(fmaxf(nv, 1e-10f));
    scale[static_cast<long long>(i) * J + j] = st;
    nrm += sum;  // vmean * red
    nrm_new += sum * st * st;
  }
  nrm = block_sum(nrm, sred);
  nrm_new = block_sum(nrm_new, sred);
  if (threadIdx.x == 0) ratio_s = sqrtf(nrm) / fmaxf(sqrtf(nrm_new), 1e-10f);
  __syncthreads();
  const float ratio = ratio_s;
  for (int j = threadIdx.x; j < J; j += blockDim.x) scale[static_cast<long long>(i) * J + j] *= ratio;
}

// p <- p - lr g - lr wd p [g p >= 0], g = X[i, r0 + r, c0 + c] * scale[i][row or col]. The parameter
// is the [rs, cs] block of the full [R, C] matrix that starts at (r0, c0) (a tensor-parallel shard,
// or the whole matrix), row-major with row stride cs. grid (chunks, n); 8 columns per thread step.
__global__ void normuon_apply_kernel(const __nv_bfloat16* __restrict__ X, const float* __restrict__ scale,
                                     const long long* __restrict__ pptrs, int R, int C, int r0, int c0, int rs, int cs,
                                     bool tall, float lr, float wd, const long long* __restrict__ peer_ptrs,
                                     int rank, int world, const uint32_t* __restrict__ status) {
  if (status_failed(status)) return;
  const int i = blockIdx.y;
  float* p = reinterpret_cast<float*>(pptrs[i]);
  // ZeRO-2 owner-computes: the owner's new values also go straight into every data-parallel peer's
  // copy of the matrix (peer_ptrs[i * world + q]), fusing the parameter all-gather into the update
  float* peer[8] = {};
  if (peer_ptrs != nullptr) {
    for (int q = 0; q < world; ++q) peer[q] = q == rank ? nullptr : reinterpret_cast<float*>(peer_ptrs[i * world + q]);
  }
  const __nv_bfloat16* Xi = X + static_cast<long long>(i) * R * C;
  const float* sc = scale + static_cast<long long>(i) * (tall ? R : C);
  const int cs8 = cs >> 3;
  const long long total = static_cast<long long>(rs) * cs8;
  const float lwd = lr * wd;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(e / cs8);
    const int c = static_cast<int>(e - static_cast<long long>(r) * cs8) << 3;
    const uint4 xv = *reinterpret_cast<const uint4*>(Xi + static_cast<long long>(r0 + r) * C + c0 + c);
    const __nv_bfloat162* xh = reinterpret_cast<const __nv_bfloat162*>(&xv);
    float4* pp = reinterpret_cast<float4*>(p + static_cast<long long>(r) * cs + c);
    float4 pa = pp[0], pb = pp[1];
    float* pv[2] = {&pa.x, &pb.x};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 f = __bfloat1622float2(xh[k >> 1]);
      const float x = (k & 1) ? f.y : f.x;
      const float s = tall ? sc[r0 + r] : sc[c0 + c + k];
      const float g = x * s;
      float& w = pv[k >> 2][k & 3];
      w = w - lr * g - ((g * w >= 0.f) ? lwd * w : 0.f);
    }
    pp[0] = pa;
    pp[1] = pb;
    if (peer_ptrs != nullptr) {
      const long long o = static_cast<long long>(r) * cs + c;
      for (int q = 0; q < world; ++q) {
        if (peer[q] == nullptr) continue;
        float4* d = reinterpret_cast<float4*>(peer[q] + o);
        d[0] = pa;
        d[1] = pb;
      }
    }
  }
}

// Sum of squares over a table of fp32 pieces (pointers and lengths), accumulated into out[0]. One
// block per row: callers split long segments into pieces of similar size (kPieceElems), so the
// work is balanced however unequal the tensors are.
__global__ void sumsq_multi_kernel(const long long* __restrict__ ptrs, const long long* __restrict__ sizes,
                                   float* __restrict__ out) {
  __shared__ float red[32];
  const float* x = reinterpret_cast<const float*>(ptrs[blockIdx.x]);
  const long long n = sizes[blockIdx.x];
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
  float acc = 0.f;
  long long start = 0;
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const long long n4 = n >> 2;
    for (long long e = threadIdx.x; e < n4; e += blockDim.x) {
      const float4 v = x4[e];
      acc = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, acc))));
    }
    start = n4 << 2;
  }
  for (long long e = start + threadIdx.x; e < n; e += blockDim.x) acc = fmaf(x[e], x[e], acc);
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) atomicAdd(out, acc);
}

// coef = min(1, max_norm / (sqrt(sumsq) + 1e-6)); norm = sqrt(sumsq)
__global__ void clip_coef_kernel(const float* __restrict__ sumsq, float max_norm, float* __restrict__ coef,
                                 float* __restrict__ norm) {
  const float nv = sqrtf(*sumsq);
  *norm = nv;
  *coef = fminf(1.f, max_norm / (nv + 1e-6f));
}

// bf16 copies of fp32 pieces: dst[k] = bf16(src[k]) for every (src, dst, size) row of the table,
// one block per row (long segments are split into pieces of similar size by the caller).
__global__ void cast_multi_kernel(const long long* __restrict__ src, const long long* __restrict__ dst,
                                  const long long* __restrict__ sizes) {
  const float* s = reinterpret_cast<const float*>(src[blockIdx.x]);
  __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(dst[blockIdx.x]);
  const long long n = sizes[blockIdx.x];
  const bool vec = ((reinterpret_cast<uintptr_t>(s) & 15u) == 0) && ((reinterpret_cast<uintptr_t>(d) & 7u) == 0);
  long long start = 0;
  if (vec) {
    const long long n4 = n >> 2;
    const float4* s4 = reinterpret_cast<const float4*>(s);
    uint2* d4 = reinterpret_cast<uint2*>(d);
    for (long long e = threadIdx.x; e < n4; e += blockDim.x) {
      const float4 v = s4[e];
      d4[e] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
    }
    start = n4 << 2;
  }
  for (long long e = start + threadIdx.x; e < n; e += blockDim.x) d[e] = __float2bfloat16_rn(s[e]);
}

int chunks_for(long long work, int dev, int ys) {
  const long long want = (work + kThreads - 1) / kThreads;
  const long long cap = std::max<long long>(1, static_cast<long long>(num_sms(dev)) * 8 / std::max(1, ys));
  return static_cast<int>(std::max<long long>(1, std::min(want, cap)));
}

void check_ptr_table(const at::Tensor& t, int64_t n, const char* name) {
  check_contig(t, name);
  MINT_CHECK(t.scalar_type() == at::kLong && t.numel() == n, name, " must be an int64 table of ", n, " pointers");
}

}  // namespace

void normuon_prep(const at::Tensor& gptrs, at::Tensor& mb, at::Tensor& sumsq, int64_t per, double mu,
                  const c10::optional<at::Tensor>& gscale) {
  const int64_t n = sumsq.numel();
  check_ptr_table(gptrs, n, "gptrs");
  check_contig(mb, "mb");
  check_contig(sumsq, "sumsq");
  MINT_CHECK(mb.scalar_type() == at::kFloat && mb.numel() == n * per && per % 4 == 0, "bad momentum stack");
  MINT_CHECK(reinterpret_cast<uintptr_t>(mb.data_ptr()) % 16 == 0, "momentum stack must be 16-byte aligned");
  const float* gs = nullptr;
  if (gscale.has_value()) {
    check_contig(*gscale, "gscale");
    gs = gscale->data_ptr<float>();
  }
  if (n == 0) return;
  c10::cuda::CUDAGuard g(mb.device());
  const int dev = mb.get_device();
  auto stream = at::cuda::getCurrentCUDAStream();
  MINT_CUDA_CHECK(cudaMemsetAsync(sumsq.data_ptr<float>(), 0, n * sizeof(float), stream));
  dim3 grid(chunks_for(per / 4, dev, static_cast<int>(n)), static_cast<unsigned>(n));
  normuon_prep_kernel<<<grid, kThreads, 0, stream>>>(reinterpret_cast<const long long*>(gptrs.data_ptr<int64_t>()),
                                                     mb.data_ptr<float>(), sumsq.data_ptr<float>(), per,
                                                     static_cast<float>(mu), gs, status_ptr(dev));
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch(2);  // the memset of sumsq and the kernel
}

void normuon_cast(const at::Tensor& gptrs, const at::Tensor& sumsq, at::Tensor& X) {
  const int64_t n = sumsq.numel();
  check_ptr_table(gptrs, n, "gptrs");
  check_contig(X, "X");
  MINT_CHECK(X.scalar_type() == at::kBFloat16 && X.dim() == 3 && X.size(0) == n, "X must be bf16 [n, R, C]");
  const long long per = X.size(1) * X.size(2);
  MINT_CHECK(per % 8 == 0, "matrix size must be a multiple of 8");
  if (n == 0) return;
  c10::cuda::CUDAGuard g(X.device());
  const int dev = X.get_device();
  dim3 grid(chunks_for(per / 8, dev, static_cast<int>(n)), static_cast<unsigned>(n));
  normuon_cast_kernel<<<grid, kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const long long*>(gptrs.data_ptr<int64_t>()), sumsq.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(X.data_ptr()), per);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

// partial sums of squares of X per row (tall: R >= C) or per column (wide); returns [S, n, J]
at::Tensor normuon_stats(const at::Tensor& X, bool tall) {
  check_contig(X, "X");
  MINT_CHECK(X.scalar_type() == at::kBFloat16 && X.dim() == 3, "X must be bf16 [n, R, C]");
  const int n = static_cast<int>(X.size(0)), R = static_cast<int>(X.size(1)), C = static_cast<int>(X.size(2));
  MINT_CHECK(C % 8 == 0, "columns must be a multiple of 8");
  c10::cuda::CUDAGuard g(X.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  if (tall) {
    auto out = at::empty({1, n, R}, X.options().dtype(at::kFloat));
    dim3 grid((R + 7) / 8, n);
    normuon_rowstats_kernel<<<grid, kThreads, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(X.data_ptr()),
                                                           out.data_ptr<float>(), R, C);
    MINT_CUDA_CHECK(cudaGetLastError());
    count_launch();
    return out;
  }
  const int colblocks = (C + 2 * kThreads - 1) / (2 * kThreads);
  const int S = std::max(1, std::min(16, num_sms(X.get_device()) * 2 / std::max(1, colblocks * n)));
  auto out = at::empty({S, n, C}, X.options().dtype(at::kFloat));
  dim3 grid(colblocks, n, S);
  normuon_colstats_kernel<<<grid, kThreads, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(X.data_ptr()),
                                                         out.data_ptr<float>(), R, C, n);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return out;
}

void normuon_scale(const at::Tensor& partial, at::Tensor& v2, at::Tensor& scale, int64_t red, double beta2) {
  check_contig(partial, "partial");
  check_contig(v2, "v2");
  check_contig(scale, "scale");
  MINT_CHECK(partial.dim() == 3, "partial must be [S, n, J]");
  const int S = static_cast<int>(partial.size(0)), n = static_cast<int>(partial.size(1));
  const int J = static_cast<int>(partial.size(2));
  MINT_CHECK(v2.numel() == static_cast<int64_t>(n) * J && scale.numel() == v2.numel(), "v2 / scale size mismatch");
  if (n == 0) return;
  c10::cuda::CUDAGuard g(partial.device());
  normuon_scale_kernel<<<n, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      partial.data_ptr<float>(), v2.data_ptr<float>(), scale.data_ptr<float>(), n, J, S, static_cast<float>(red),
      static_cast<float>(beta2), status_ptr(partial.get_device()));
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void normuon_apply(const at::Tensor& X, const at::Tensor& scale, const at::Tensor& pptrs, int64_t r0, int64_t c0,
                   int64_t rs, int64_t cs, bool tall, double lr, double wd, const c10::optional<at::Tensor>& peer_ptrs,
                   int64_t rank, int64_t world) {
  check_contig(X, "X");
  check_contig(scale, "scale");
  const int n = static_cast<int>(X.size(0)), R = static_cast<int>(X.size(1)), C = static_cast<int>(X.size(2));
  check_ptr_table(pptrs, n, "pptrs");
  MINT_CHECK(cs % 8 == 0 && c0 % 8 == 0, "shard columns must be multiples of 8");
  MINT_CHECK(r0 + rs <= R && c0 + cs <= C, "shard outside the matrix");
  const bool push = peer_ptrs.has_value() && peer_ptrs->defined();
  if (push) {
    MINT_CHECK(world >= 2 && world <= 8 && rank >= 0 && rank < world, "normuon_apply: push needs 2..8 ranks");
    check_ptr_table(*peer_ptrs, static_cast<int64_t>(n) * world, "peer_ptrs");
  }
  if (n == 0 || rs == 0) return;
  c10::cuda::CUDAGuard g(X.device());
  const int dev = X.get_device();
  dim3 grid(chunks_for(rs * cs / 8, dev, n), static_cast<unsigned>(n));
  normuon_apply_kernel<<<grid, kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(X.data_ptr()), scale.data_ptr<float>(),
      reinterpret_cast<const long long*>(pptrs.data_ptr<int64_t>()), R, C, static_cast<int>(r0), static_cast<int>(c0),
      static_cast<int>(rs), static_cast<int>(cs), tall, static_cast<float>(lr), static_cast<float>(wd),
      push ? reinterpret_cast<const long long*>(peer_ptrs->data_ptr<int64_t>()) : nullptr, static_cast<int>(rank),
      static_cast<int>(world), status_ptr(dev));
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

// out[0] += sum of squares of every piece (out is not cleared here); one block per table row
void sumsq_multi(const at::Tensor& ptrs, const at::Tensor& sizes, at::Tensor& out, int64_t max_len) {
  const int64_t n = ptrs.numel();
  check_ptr_table(ptrs, n, "ptrs");
  check_ptr_table(sizes, n, "sizes");
  check_contig(out, "out");
  (void)max_len;
  if (n == 0) return;
  c10::cuda::CUDAGuard g(out.device());
  sumsq_multi_kernel<<<static_cast<unsigned>(n), kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const long long*>(ptrs.data_ptr<int64_t>()),
      reinterpret_cast<const long long*>(sizes.data_ptr<int64_t>()), out.data_ptr<float>());
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void clip_coef(const at::Tensor& sumsq, double max_norm, at::Tensor& coef, at::Tensor& norm) {
  check_contig(sumsq, "sumsq");
  check_contig(coef, "coef");
  check_contig(norm, "norm");
  c10::cuda::CUDAGuard g(sumsq.device());
  clip_coef_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(sumsq.data_ptr<float>(), static_cast<float>(max_norm),
                                                                   coef.data_ptr<float>(), norm.data_ptr<float>());
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void cast_multi(const at::Tensor& src, const at::Tensor& dst, const at::Tensor& sizes, int64_t max_len) {
  const int64_t n = src.numel();
  check_ptr_table(src, n, "src");
  check_ptr_table(dst, n, "dst");
  check_ptr_table(sizes, n, "sizes");
  (void)max_len;
  if (n == 0) return;
  c10::cuda::CUDAGuard g(src.device());
  cast_multi_kernel<<<static_cast<unsigned>(n), kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const long long*>(src.data_ptr<int64_t>()),
      reinterpret_cast<const long long*>(dst.data_ptr<int64_t>()),
      reinterpret_cast<const long long*>(sizes.data_ptr<int64_t>()));
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

}  // namespace mint
