// FlashAttention backward for sm_100a on tcgen05 tensor cores (head_dim 128, bf16, GQA).
//
// One CTA per (128-key tile, KV head, batch) loops over every query head that shares the KV
// head and over the query tiles inside the causal / sliding-window band, so dK and dV accumulate
// in tensor memory without atomics. Per query tile (all operands from shared memory, fp32 TMEM
// accumulators, 256 threads: warp 0 TMA, warp 1 MMA issue, warps 4..7 math):
//   S^T  = K Q^T            -> TMEM [0,128)     (rows = keys)
//   dP^T = V dO^T           -> TMEM [128,256)
//   P^T  = exp(S^T*scale - lse),  dS^T = P^T * (dP^T - D)      (math warps, one key row each)
//   dV  += P^T dO           -> TMEM [256,384)   (P^T K-major, dO read MN-major)
//   dK  += dS^T Q           -> TMEM [384,512)   (Q read MN-major)
//   dQ_i = dS K             -> TMEM [0,128)     (dS^T read MN-major as the A operand; K MN-major)
// The same shared-memory bytes serve as K-major and MN-major operands: a TMA box of 64 head dims
// x 128 rows with 128B swizzle is the canonical layout for both. dQ is accumulated across key tiles
// with 16-byte fp32 vector reductions into an fp32 buffer; a final pass converts it to bf16.
// D_i = rowsum(dO_i * O_i) is computed by a preprocessing kernel. All waits are bounded.
//
// Pipelining: Q / dO stream through a 2-stage ring; P and dS share one shared-memory tile (dS is
// written once dV has consumed P); dQ_i lands in the dP^T columns once dS is computed, so the MMA
// issue order dV_i, S_{i+1}, dK_i, dQ_i, dP_{i+1} keeps the tensor pipe busy while the math warps
// produce dS_i and drain dQ_i.
#include <cstdio>
#include <cstdlib>

#include "common.cuh"
#include "host_common.h"
#include "attention_bwd_raw.h"

namespace mint {

const int2* doc_bounds_ptr(const c10::optional<at::Tensor>& doc, const c10::optional<at::Tensor>& dbounds,
                           int64_t B, int64_t T, at::Tensor& holder);

namespace fab {

constexpr int kB = 128;  // rows per tile (keys or queries)
constexpr int kD = 128;
constexpr int kThreads = 384;  // warp 0 TMA, warp 1 MMA, warps 4..11 math (2 per TMEM lane quadrant)
constexpr int kTileBytes = kB * kD * 2;
constexpr int kAtomBytes = kTileBytes / 2;

struct BwdParams {
  float* dq_acc;          // [B, T, Hq, D] fp32 (zero-initialized)
  __nv_bfloat16* dk;      // [B, T, Hkv, D]
  __nv_bfloat16* dv;      // [B, T, Hkv, D]
  const float* lse;       // [B, Hq, T] natural log
  const float* delta;     // [B, Hq, T]
  const int* doc;         // [B, T] or null
  const int2* dbounds;    // [B, T] document run [start, end) per token; start < 0: row not sorted
  int B, T, Hq, Hkv;
  int causal, window;
  float scale, scale_log2;
  uint32_t* status;
  // MINT_FA_TRACE=1: clock64 stamps of block (0, 0, 0) -- key tile 0, the one with the most query
  // tiles under a causal mask -- for the first kTraceTiles query tiles: [tile][kTraceSteps] from
  // lane 0 of math warp 4, then [tile][4] from the MMA thread (diagnostics only; null otherwise)
  unsigned long long* trace;
};
constexpr int kTraceTiles = 64;
constexpr int kTraceSteps = 12;

struct Smem {
  uint8_t k[kTileBytes];
  uint8_t v[kTileBytes];
  uint8_t q[2][kTileBytes];
  uint8_t dout[2][kTileBytes];
  uint8_t pds[kTileBytes];  // P^T, then dS^T of the same query tile
  uint64_t kv_full, q_full[2], q_empty[2], do_full[2], do_empty[2];
  uint64_t s_full, dp_full, p_ready, dv_done, ds_ready, dq_full, dq_free, mma_done;
  uint32_t tmem_base;
  int abort_flag;
};
// dynamic shared memory = the struct + 1024 bytes of alignment slack; 232448 is the per-block opt-in limit
static_assert(sizeof(Smem) + 1024 <= 232448, "shared-memory layout exceeds the per-block limit");


// K-major operand (row-contiguous 128 x 128 tile, 2 atoms along K): descriptor of K-step k
__device__ __forceinline__ uint64_t kmaj(uint32_t base, int k) {
  return umma_desc_sw128(base + (k >> 2) * kAtomBytes + (k & 3) * 32, 16, 1024);
}
// the same tile read MN-major (its rows are the contraction dim): K-step k = 16 rows
__device__ __forceinline__ uint64_t mnmaj(uint32_t base, int k) {
  return umma_desc_sw128(base + k * 2048, kAtomBytes, 1024);
}

__device__ __forceinline__ void mma_kk(uint32_t d, uint32_t a, uint32_t b, bool acc) {
  constexpr uint32_t idesc = umma_idesc_bf16(kB, kB, false, false);
#pragma unroll
  for (int k = 0; k < 8; ++k) umma_bf16(d, kmaj(a, k), kmaj(b, k), idesc, (acc || k > 0) ? 1u : 0u);
}
__device__ __forceinline__ void mma_kmn(uint32_t d, uint32_t a, uint32_t b, bool acc) {
  constexpr uint32_t idesc = umma_idesc_bf16(kB, kD, false, true);
#pragma unroll
  for (int k = 0; k < 8; ++k) umma_bf16(d, kmaj(a, k), mnmaj(b, k), idesc, (acc || k > 0) ? 1u : 0u);
}
__device__ __forceinline__ void mma_mnmn(uint32_t d, uint32_t a, uint32_t b, bool acc) {
  constexpr uint32_t idesc = umma_idesc_bf16(kB, kD, true, true);
#pragma unroll
  for (int k = 0; k < 8; ++k) umma_bf16(d, mnmaj(a, k), mnmaj(b, k), idesc, (acc || k > 0) ? 1u : 0u);
}

// 64 columns (one swizzle atom `a`) of row r of a K-major 128B-swizzled bf16 tile from finite fp32
// values (P or dS; converted on the integer pipe, which the exponentials do not use)
__device__ __forceinline__ void store_half_row_sw128(uint8_t* tile, int a, int r, const float (&x)[64]) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int e = c * 8;
    uint4 v4 = make_uint4(pack_bf16x2_int(x[e], x[e + 1]), pack_bf16x2_int(x[e + 2], x[e + 3]),
                          pack_bf16x2_int(x[e + 4], x[e + 5]), pack_bf16x2_int(x[e + 6], x[e + 7]));
    *reinterpret_cast<uint4*>(tile + a * kAtomBytes + r * 128 + ((c ^ (r & 7)) << 4)) = v4;
  }
}

// 64 columns (one swizzle atom `a`) of row r of a K-major 128B-swizzled bf16 tile, already packed
__device__ __forceinline__ void store_half_row_packed(uint8_t* tile, int a, int r, const uint32_t (&pk)[32]) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    *reinterpret_cast<uint4*>(tile + a * kAtomBytes + r * 128 + ((c ^ (r & 7)) << 4)) =
        make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
  }
}

__device__ __forceinline__ void load_row64(uint32_t taddr, float (&x)[64]) {
  uint32_t u0[32], u1[32];  // both loads in flight under one wait
  tmem_ld_32x32b_x32(taddr, u0);
  tmem_ld_32x32b_x32(taddr + 32, u1);
  tmem_ld_wait();
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    x[e] = __uint_as_float(u0[e]);
    x[32 + e] = __uint_as_float(u1[e]);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                  const __grid_constant__ CUtensorMap tdq, BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = p.Hq / p.Hkv;
  const int k0 = kt * kB;
  const int ntq = (p.T + kB - 1) / kB;
  const int2* db = p.dbounds != nullptr ? p.dbounds + static_cast<long long>(b) * p.T : nullptr;
  const int k_last = min(p.T, k0 + kB) - 1;
  int i0 = p.causal ? k0 / kB : 0;
  int i1 = ntq;
  if (p.window >= 0) i1 = min(ntq, (k0 + kB - 1 + p.window) / kB + 1);
  // doc_sorted: document masks come from the [start, end) bounds; else (ids given without bounds,
  // or an unsorted row) ids are compared per element and no tile is skipped for documents
  const bool doc_sorted = db != nullptr && db[k0].x >= 0;
  if (doc_sorted) {
    // queries outside the documents of this key tile never attend to it
    i0 = max(i0, db[k0].x / kB);
    i1 = min(i1, (db[k_last].y + kB - 1) / kB);
  }
  const int nq = max(0, i1 - i0);
  const int n = G * nq;
  volatile int* abort_flag = &s.abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&s.kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.q_full[i], 1);
      mbar_init(&s.q_empty[i], 1);
      mbar_init(&s.do_full[i], 1);
      mbar_init(&s.do_empty[i], 8);  // the math warps, once their dQ staging in it has been read
    }
    mbar_init(&s.s_full, 1);
    mbar_init(&s.dp_full, 1);
    mbar_init(&s.p_ready, 8);
    mbar_init(&s.dv_done, 1);
    mbar_init(&s.ds_ready, 8);
    mbar_init(&s.dq_full, 1);
    mbar_init(&s.dq_free, 8);
    mbar_init(&s.mma_done, 1);
    s.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&s.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  // dQ_i reuses the dP^T columns once dS_i has been computed from them
  const uint32_t t_s = tmem, t_dp = tmem + 128, t_dq = tmem + 128, t_dv = tmem + 256, t_dk = tmem + 384;

  if (warp == 0) {
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      tma_prefetch_desc(&tdo);
      const int krow = b * p.T + k0;
      mbar_arrive_expect_tx(&s.kv_full, 2 * kTileBytes);
      tma_load_3d(s.k, &tk, &s.kv_full, 0, hk, krow);
      tma_load_3d(s.k + kAtomBytes, &tk, &s.kv_full, 64, hk, krow);
      tma_load_3d(s.v, &tv, &s.kv_full, 0, hk, krow);
      tma_load_3d(s.v + kAtomBytes, &tv, &s.kv_full, 64, hk, krow);
      for (int it = 0; it < n; ++it) {
        const int h = hk * G + it / nq;
        const int qrow = b * p.T + (i0 + it % nq) * kB;
        const int st = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (!mbar_wait(&s.q_empty[st], ph ^ 1u, p.status, kStatusTimeoutAttention, abort_flag)) break;
        mbar_arrive_expect_tx(&s.q_full[st], kTileBytes);
        tma_load_3d(s.q[st], &tq, &s.q_full[st], 0, h, qrow);
        tma_load_3d(s.q[st] + kAtomBytes, &tq, &s.q_full[st], 64, h, qrow);
        if (!mbar_wait(&s.do_empty[st], ph ^ 1u, p.status, kStatusTimeoutAttention, abort_flag)) break;
        mbar_arrive_expect_tx(&s.do_full[st], kTileBytes);
        tma_load_3d(s.dout[st], &tdo, &s.do_full[st], 0, h, qrow);
        tma_load_3d(s.dout[st] + kAtomBytes, &tdo, &s.do_full[st], 64, h, qrow);
      }
      if (*abort_flag) {
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n > 0) {
      const uint32_t a_k = smem_u32(s.k), a_v = smem_u32(s.v), a_pds = smem_u32(s.pds);
      bool ok = mbar_wait(&s.kv_full, 0, p.status, kStatusTimeoutAttention, abort_flag) &&
                mbar_wait(&s.q_full[0], 0, p.status, kStatusTimeoutAttention, abort_flag) &&
                mbar_wait(&s.do_full[0], 0, p.status, kStatusTimeoutAttention, abort_flag);
      if (ok) {
        tc_fence_after();
        mma_kk(t_s, a_k, smem_u32(s.q[0]), false);      // S^T_0 = K Q_0^T
        umma_commit(&s.s_full);
        mma_kk(t_dp, a_v, smem_u32(s.dout[0]), false);  // dP^T_0 = V dO_0^T
        umma_commit(&s.dp_full);
      }
      unsigned long long* tr = (p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
                                   ? p.trace + kTraceTiles * kTraceSteps
                                   : nullptr;
      for (int it = 0; it < n && ok; ++it) {
        const int st = it & 1;
        const uint32_t ph = it & 1;
        const uint32_t a_q = smem_u32(s.q[st]), a_do = smem_u32(s.dout[st]);
        if (tr != nullptr && it < kTraceTiles) tr[it * 4] = clock64();
        if (!(ok = mbar_wait(&s.p_ready, ph, p.status, kStatusTimeoutAttention, abort_flag))) break;
        if (tr != nullptr && it < kTraceTiles) tr[it * 4 + 1] = clock64();
        tc_fence_after();
        mma_kmn(t_dv, a_pds, a_do, it > 0);  // dV += P^T dO
        umma_commit(&s.dv_done);
        const bool more = it + 1 < n;
        if (more) {
          const int sn = (it + 1) & 1;
          const uint32_t pn = ((it + 1) >> 1) & 1;
          if (!(ok = mbar_wait(&s.q_full[sn], pn, p.status, kStatusTimeoutAttention, abort_flag))) break;
          tc_fence_after();
          mma_kk(t_s, a_k, smem_u32(s.q[sn]), false);  // S^T_{i+1}: S_i was consumed before p_ready_i
          umma_commit(&s.s_full);
        }
        if (!(ok = mbar_wait(&s.ds_ready, ph, p.status, kStatusTimeoutAttention, abort_flag))) break;
        if (tr != nullptr && it < kTraceTiles) tr[it * 4 + 2] = clock64();
        tc_fence_after();
        mma_kmn(t_dk, a_pds, a_q, it > 0);  // dK += dS^T Q
        mma_mnmn(t_dq, a_pds, a_k, false);  // dQ_i = dS K (dP^T_i was consumed before ds_ready_i)
        umma_commit(&s.dq_full);
        umma_commit(&s.q_empty[st]);  // dO_i's buffer is released by the math warps (dQ staging)
        if (more) {
          const int sn = (it + 1) & 1;
          const uint32_t pn = ((it + 1) >> 1) & 1;
          if (!(ok = mbar_wait(&s.do_full[sn], pn, p.status, kStatusTimeoutAttention, abort_flag))) break;
          if (!(ok = mbar_wait(&s.dq_free, ph, p.status, kStatusTimeoutAttention, abort_flag))) break;
          if (tr != nullptr && it < kTraceTiles) tr[it * 4 + 3] = clock64();
          tc_fence_after();
          mma_kk(t_dp, a_v, smem_u32(s.dout[sn]), false);  // dP^T_{i+1}
          umma_commit(&s.dp_full);
        }
      }
      umma_commit(&s.mma_done);
      mbar_wait(&s.mma_done, 0, p.status, kStatusTimeoutAttention, nullptr);
    }
  } else if (warp >= 4) {
    // warp 4 + 4h + q: TMEM lane quadrant q (rows q*32 .. q*32+31), columns [64h, 64h + 64)
    const int q = warp & 3;
    const int half = (warp - 4) >> 2;
    const int cb = half * 64;
    const int r = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int kj = k0 + r;
    const int doc_k = (p.doc != nullptr && kj < p.T) ? p.doc[static_cast<long long>(b) * p.T + kj] : 0;
    const int2 dk = (doc_sorted && kj < p.T) ? db[kj] : make_int2(0, p.T);
    bool ok = n > 0;
    unsigned long long* tr = (p.trace != nullptr && lane == 0 && warp == 4 && blockIdx.x == 0 && blockIdx.y == 0 &&
                              blockIdx.z == 0)
                                 ? p.trace
                                 : nullptr;
#define FAB_STAMP(k) \
  if (tr != nullptr && it < kTraceTiles) tr[it * kTraceSteps + (k)] = clock64();
    for (int it = 0; it < n && ok; ++it) {
      FAB_STAMP(0)
      const uint32_t ph = it & 1;
      const int h = hk * G + it / nq;
      const int q0 = (i0 + it % nq) * kB;
      const int q_last = min(p.T, q0 + kB) - 1;
      // this query tile's LSE (natural log) and delta rows, read straight from global memory (every
      // lane of a warp reads the same 64 values: broadcast loads, L1-resident after the first warp);
      // columns past T read the row's last valid value (their probabilities are masked to 0)
      const long long rowbase = (static_cast<long long>(b) * p.Hq + h) * p.T + q0 + cb;
      const float* lse_row = p.lse + rowbase;
      const float* dlt_row = p.delta + rowbase;
      const bool full_cols = q0 + cb + 64 <= p.T;
      const int last_col = p.T - 1 - (q0 + cb);
      // this tile's LSE pairs, loaded before the S wait so their latency hides behind it
      float2 lse_pk[32];
      if (full_cols) {
#pragma unroll
        for (int c = 0; c < 32; ++c) lse_pk[c] = __ldg(reinterpret_cast<const float2*>(lse_row) + c);
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          lse_pk[c] = make_float2(__ldg(lse_row + min(2 * c, last_col)), __ldg(lse_row + min(2 * c + 1, last_col)));
        }
      }
      FAB_STAMP(1)
      if (!(ok = mbar_wait_warp(&s.s_full, ph, p.status, kStatusTimeoutAttention, abort_flag))) break;
      FAB_STAMP(2)
      tc_fence_after();
      float x[64];
      load_row64(t_s + lane_off + cb, x);
      FAB_STAMP(3)
      const int lo_i = min(k0, q0), hi_i = max(k_last, q_last);
      const bool doc_mask = p.doc != nullptr && !(doc_sorted && db[lo_i].y > hi_i);
      const bool need_mask = (p.causal && k0 + kB - 1 > q0) || (p.window >= 0 && q0 + kB - 1 - k0 > p.window) ||
                             q0 + kB > p.T || k0 + kB > p.T || doc_mask;
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const int qi = q0 + cb + c;
          bool keep = qi < p.T && kj < p.T && qi >= dk.x && qi < dk.y;
          if (p.causal) keep = keep && kj <= qi;
          if (p.window >= 0) keep = keep && qi - kj <= p.window;
          if (p.doc != nullptr && !doc_sorted && keep) keep = p.doc[static_cast<long long>(b) * p.T + qi] == doc_k;
          if (!keep) x[c] = -INFINITY;
        }
      }
      // P^T = exp2(S^T * scale - lse), two elements per instruction (packed fp32 FMA, bf16x2 MUFU
      // exponential straight into the bf16 operand layout); masked entries give 2^-inf = 0
      uint32_t pk[32];
      {
        const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
        const float2 nl2e = make_float2(-1.4426950408889634f, -1.4426950408889634f);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float2 t = ffma2(make_float2(x[2 * c], x[2 * c + 1]), sc2, fmul2(lse_pk[c], nl2e));
          pk[c] = ex2_bf16x2(t.x, t.y);
        }
      }
      FAB_STAMP(4)
      // the shared P/dS tile is free: dK_{i-1} / dQ_{i-1} (dq_full_{i-1}) finished reading dS_{i-1}, and
      // this warp's dQ_{i-1} reduce-adds (staged in the same bytes it now writes, and in dO_{i-1}'s
      // buffer, which is released to the producer here) read their sources
      if (lane == 0) {
        bulk_wait_read<0>();
        if (it > 0) mbar_arrive(&s.do_empty[(it - 1) & 1]);
      }
      __syncwarp();
      store_half_row_packed(s.pds, half, r, pk);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.p_ready);
      // this tile's delta pairs, loaded before the dP wait
      float2 dlt_pk[32];
      if (full_cols) {
#pragma unroll
        for (int c = 0; c < 32; ++c) dlt_pk[c] = __ldg(reinterpret_cast<const float2*>(dlt_row) + c);
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          dlt_pk[c] = make_float2(__ldg(dlt_row + min(2 * c, last_col)), __ldg(dlt_row + min(2 * c + 1, last_col)));
        }
      }
      FAB_STAMP(5)
      if (!(ok = mbar_wait_warp(&s.dp_full, ph, p.status, kStatusTimeoutAttention, abort_flag))) break;
      FAB_STAMP(6)
      tc_fence_after();
      // dS^T = P^T (dP^T - delta), in packed fp32 pairs from the bf16 P the dV MMA used
      {
        uint32_t u0[32], u1[32];  // both loads in flight under one wait
        tmem_ld_32x32b_x32(t_dp + lane_off + cb, u0);
        tmem_ld_32x32b_x32(t_dp + lane_off + cb + 32, u1);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const uint32_t* u = c < 16 ? u0 : u1;
          const int e = (2 * c) & 31;
          const float2 d2 = dlt_pk[c];
          const float2 g = fadd2(make_float2(__uint_as_float(u[e]), __uint_as_float(u[e + 1])),
                                 make_float2(-d2.x, -d2.y));
          const float2 ds = fmul2(bf16x2_to_float2(pk[c]), g);
          pk[c] = pack_bf16x2(ds.x, ds.y);
        }
      }
      FAB_STAMP(7)
      // dS overwrites P only after dV has consumed it
      if (!(ok = mbar_wait_warp(&s.dv_done, ph, p.status, kStatusTimeoutAttention, abort_flag))) break;
      FAB_STAMP(8)
      store_half_row_packed(s.pds, half, r, pk);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.ds_ready);
      FAB_STAMP(9)
      if (!(ok = mbar_wait_warp(&s.dq_full, ph, p.status, kStatusTimeoutAttention, abort_flag))) break;
      FAB_STAMP(10)
      tc_fence_after();
      // dQ rows: TMEM lane = query index within the tile; this warp drains 64 of the 128 head dims.
      // The P/dS tile and dO_i's buffer are free now (the dK / dQ MMAs that read dS completed, and
      // before them dV_i, the last reader of dO_i): each warp stages its two 32 rows x 32 columns
      // boxes of dQ in its own 4 KB of each and reduce-adds them into the fp32 accumulator with one
      // TMA bulk reduction per box; nothing waits for those reads until the next tile.
      {
        uint32_t u0[32], u1[32];  // both loads in flight under one wait
        tmem_ld_32x32b_x32(t_dq + lane_off + cb, u0);
        tmem_ld_32x32b_x32(t_dq + lane_off + cb + 32, u1);
        tmem_ld_wait();
        uint8_t* stage0 = s.pds + (warp - 4) * 4096;
        uint8_t* stage1 = s.dout[it & 1] + (warp - 4) * 4096;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int off = lane * 128 + ((j ^ (lane & 7)) << 4);
          *reinterpret_cast<float4*>(stage0 + off) =
              make_float4(__uint_as_float(u0[4 * j]) * p.scale, __uint_as_float(u0[4 * j + 1]) * p.scale,
                          __uint_as_float(u0[4 * j + 2]) * p.scale, __uint_as_float(u0[4 * j + 3]) * p.scale);
          *reinterpret_cast<float4*>(stage1 + off) =
              make_float4(__uint_as_float(u1[4 * j]) * p.scale, __uint_as_float(u1[4 * j + 1]) * p.scale,
                          __uint_as_float(u1[4 * j + 2]) * p.scale, __uint_as_float(u1[4 * j + 3]) * p.scale);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_4d(&tdq, stage0, cb, h, q0 + q * 32, b);  // rows past T are clipped
          tma_reduce_add_4d(&tdq, stage1, cb + 32, h, q0 + q * 32, b);
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.dq_free);
      FAB_STAMP(11)
    }
#undef FAB_STAMP
    // the dQ reductions have read their shared-memory sources before it is released (their global
    // writes complete with the grid, before any later kernel on the stream reads dQ)
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
    // dK / dV rows: TMEM lane = key index (tcgen05.ld is warp-collective: every lane loads)
    ok = __all_sync(0xffffffffu, ok);
    const bool key_ok = kj < p.T;
    __nv_bfloat16* dkr = p.dk + ((static_cast<long long>(b) * p.T + (key_ok ? kj : 0)) * p.Hkv + hk) * kD + cb;
    __nv_bfloat16* dvr = p.dv + ((static_cast<long long>(b) * p.T + (key_ok ? kj : 0)) * p.Hkv + hk) * kD + cb;
    if (ok && n > 0) {
      tc_fence_after();
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        uint32_t uk[32], uv[32];
        tmem_ld_32x32b_x32(t_dk + lane_off + cb + c2 * 32, uk);
        tmem_ld_32x32b_x32(t_dv + lane_off + cb + c2 * 32, uv);
        tmem_ld_wait();
        if (!key_ok) continue;
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 a, v;
          a.x = pack_bf16x2(__uint_as_float(uk[e]) * p.scale, __uint_as_float(uk[e + 1]) * p.scale);
          a.y = pack_bf16x2(__uint_as_float(uk[e + 2]) * p.scale, __uint_as_float(uk[e + 3]) * p.scale);
          a.z = pack_bf16x2(__uint_as_float(uk[e + 4]) * p.scale, __uint_as_float(uk[e + 5]) * p.scale);
          a.w = pack_bf16x2(__uint_as_float(uk[e + 6]) * p.scale, __uint_as_float(uk[e + 7]) * p.scale);
          v.x = pack_bf16x2(__uint_as_float(uv[e]), __uint_as_float(uv[e + 1]));
          v.y = pack_bf16x2(__uint_as_float(uv[e + 2]), __uint_as_float(uv[e + 3]));
          v.z = pack_bf16x2(__uint_as_float(uv[e + 4]), __uint_as_float(uv[e + 5]));
          v.w = pack_bf16x2(__uint_as_float(uv[e + 6]), __uint_as_float(uv[e + 7]));
          *reinterpret_cast<uint4*>(dkr + c2 * 32 + e) = a;
          *reinterpret_cast<uint4*>(dvr + c2 * 32 + e) = v;
        }
      }
    } else if (n == 0 && key_ok) {
      for (int c = 0; c < 64; ++c) {
        dkr[c] = __float2bfloat16_rn(0.f);
        dvr[c] = __float2bfloat16_rn(0.f);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta[b, h, i] = sum_d dO[b, i, h, d] * O[b, i, h, d]   (one warp per row)
__global__ void __launch_bounds__(256) fa_bwd_delta_kernel(const __nv_bfloat16* __restrict__ dout,
                                                           const __nv_bfloat16* __restrict__ o,
                                                           float* __restrict__ delta, int B, int T, int Hq) {
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= static_cast<long long>(B) * T * Hq) return;
  const __nv_bfloat16* a = dout + row * kD + lane * 4;
  const __nv_bfloat16* c = o + row * kD + lane * 4;
  float acc = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) acc += __bfloat162float(a[e]) * __bfloat162float(c[e]);
  acc = warp_sum(acc);
  if (lane == 0) {
    const int h = static_cast<int>(row % Hq);
    const long long bt = row / Hq;
    const int t = static_cast<int>(bt % T);
    const int bb = static_cast<int>(bt / T);
    delta[(static_cast<long long>(bb) * Hq + h) * T + t] = acc;
  }
}

__global__ void fa_cast_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, long long n4) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(src)[i];
    uint2 u;
    u.x = pack_bf16x2(v.x, v.y);
    u.y = pack_bf16x2(v.z, v.w);
    reinterpret_cast<uint2*>(dst)[i] = u;
  }
}

}  // namespace fab

// fp32 dQ accumulator [B, T, Hq, 128] as a 4-D TMA map {d, h, t, b}: reduce-add boxes of 32 rows
// (consecutive t of one head) x 32 dims, clipped at the end of each sequence.
static CUtensorMap dq_acc_map(float* dq_acc, int B, int T, int Hq) {
  const uint64_t dims[4] = {128, static_cast<uint64_t>(Hq), static_cast<uint64_t>(T), static_cast<uint64_t>(B)};
  const uint64_t strides[3] = {128, static_cast<uint64_t>(Hq) * 128, static_cast<uint64_t>(T) * Hq * 128};
  const uint32_t box[4] = {32, 1, 32, 1};
  return make_tmap_4d(dq_acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// MINT_FA_TRACE=1 diagnostics: the stamp buffer of the last backward (zeros if tracing is off)
at::Tensor& fab_trace_buffer() {
  static at::Tensor buf;
  return buf;
}

at::Tensor flash_attn_bwd_trace() {
  at::Tensor& buf = fab_trace_buffer();
  return buf.defined() ? buf.clone() : at::zeros({(fab::kTraceSteps + 4) * fab::kTraceTiles}, at::kLong);
}

std::vector<at::Tensor> flash_attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                       const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse,
                                       const c10::optional<at::Tensor>& doc, bool causal, int64_t window,
                                       double scale, const c10::optional<at::Tensor>& dbounds) {
  const at::Tensor* inputs[5] = {&dout, &q, &k, &v, &o};
  for (const at::Tensor* t : inputs) {
    check_contig(*t, "flash_attn_bwd input");
    MINT_CHECK(t->scalar_type() == at::kBFloat16, "flash_attn_bwd expects bf16");
  }
  const int B = static_cast<int>(q.size(0)), T = static_cast<int>(q.size(1));
  const int Hq = static_cast<int>(q.size(2)), Hkv = static_cast<int>(k.size(2));
  MINT_CHECK(q.size(3) == fab::kD && Hq % Hkv == 0 && dout.sizes() == q.sizes() && o.sizes() == q.sizes(),
             "flash_attn_bwd shape mismatch");
  auto dq_acc = at::zeros(q.sizes(), q.options().dtype(at::kFloat));
  auto dq = at::empty_like(q);
  auto dk = at::empty_like(k);
  auto dv = at::empty_like(v);
  auto delta = at::empty({B, Hq, T}, q.options().dtype(at::kFloat));
  if (B == 0 || T == 0) return {dq.zero_(), dk.zero_(), dv.zero_()};
  c10::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const long long rows = static_cast<long long>(B) * T * Hq;
  fab::fa_bwd_delta_kernel<<<static_cast<int>((rows * 32 + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()),
      delta.data_ptr<float>(), B, T, Hq);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();

  fab::BwdParams p{};
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  at::Tensor bounds_holder;
  if (doc.has_value() && doc->defined()) {
    check_contig(*doc, "doc_ids");
    MINT_CHECK(doc->scalar_type() == at::kInt && doc->numel() == static_cast<int64_t>(B) * T, "doc_ids must be int32 [B, T]");
    p.doc = doc->data_ptr<int>();
    p.dbounds = doc_bounds_ptr(doc, dbounds, B, T, bounds_holder);
  }
  p.B = B;
  p.T = T;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.causal = causal ? 1 : 0;
  p.window = static_cast<int>(window);
  p.scale = static_cast<float>(scale);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.status = status_ptr(q.get_device());
  static const bool fa_trace = std::getenv("MINT_FA_TRACE") != nullptr;
  if (fa_trace) {
    at::Tensor& buf = fab_trace_buffer();
    if (!buf.defined() || buf.device() != q.device()) {
      buf = at::zeros({(fab::kTraceSteps + 4) * fab::kTraceTiles}, q.options().dtype(at::kLong));
    }
    p.trace = reinterpret_cast<unsigned long long*>(buf.data_ptr<int64_t>());
  }
  auto map = [&](const at::Tensor& t, int H) {
    return make_tmap_3d_bf16(t.data_ptr(), fab::kD, H, static_cast<uint64_t>(B) * T, fab::kD,
                             static_cast<uint64_t>(H) * fab::kD, 64, 1, 128, true);
  };
  const CUtensorMap tq = map(q, Hq), tk = map(k, Hkv), tv = map(v, Hkv), tdo = map(dout, Hq);
  const CUtensorMap tdq = dq_acc_map(dq_acc.data_ptr<float>(), B, T, Hq);
  const int smem = static_cast<int>(sizeof(fab::Smem)) + 1024;
  static const bool trace = std::getenv("MINT_TRACE_LAUNCH") != nullptr;
  auto step = [&](const char* what) {
    if (!trace) return;
    const cudaError_t e = cudaDeviceSynchronize();
    std::fprintf(stderr, "[mint trace] flash_attn_bwd %s: %s (smem %d)\n", what, cudaGetErrorString(e), smem);
    std::fflush(stderr);
  };
  step("after delta kernel");
  static bool configured[64] = {};
  const int dev = q.get_device();
  if (!configured[dev & 63]) {
    check_smem_optin(smem, dev, "fa_bwd_kernel");
    MINT_CUDA_CHECK(cudaFuncSetAttribute(fab::fa_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured[dev & 63] = true;
  }
  if (trace) {
    cudaFuncAttributes fa{};
    const cudaError_t e = cudaFuncGetAttributes(&fa, fab::fa_bwd_kernel);
    std::fprintf(stderr, "[mint trace] fa_bwd_kernel attrs %s: regs %d local %zu maxThreads %d maxDynSmem %d\n",
                 cudaGetErrorString(e), fa.numRegs, fa.localSizeBytes, fa.maxThreadsPerBlock,
                 fa.maxDynamicSharedSizeBytes);
    std::fflush(stderr);
  }
  dim3 grid((T + fab::kB - 1) / fab::kB, Hkv, B);
  step("before main kernel");
  fab::fa_bwd_kernel<<<grid, fab::kThreads, smem, stream>>>(tq, tk, tv, tdo, tdq, p);
  step("after main kernel launch");
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  const long long n4 = q.numel() / 4;
  fab::fa_cast_kernel<<<static_cast<int>(std::min<long long>((n4 + 255) / 256, 148LL * 16)), 256, 0, stream>>>(
      dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), n4);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return {dq, dk, dv};
}

// Raw-pointer launch of the same three backward kernels (delta, main, dQ cast) for callers that
// own every buffer themselves; used by the allocation-free entry point in
// flash_attn_bwd_noalloc.cu. `dq_acc` must hold zeros when the first kernel runs.
void flash_attn_bwd_launch_raw(const FlashBwdRaw& a, cudaStream_t stream) {
  const long long rows = static_cast<long long>(a.B) * a.T * a.Hq;
  fab::fa_bwd_delta_kernel<<<static_cast<int>((rows * 32 + 255) / 256), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(a.dout), static_cast<const __nv_bfloat16*>(a.o), a.delta, a.B, a.T, a.Hq);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  fab::BwdParams p{};
  p.dq_acc = a.dq_acc;
  p.dk = static_cast<__nv_bfloat16*>(a.dk);
  p.dv = static_cast<__nv_bfloat16*>(a.dv);
  p.lse = a.lse;
  p.delta = a.delta;
  p.doc = a.doc;
  p.B = a.B;
  p.T = a.T;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.causal = a.causal ? 1 : 0;
  p.window = a.window;
  p.scale = a.scale;
  p.scale_log2 = static_cast<float>(static_cast<double>(a.scale) * 1.4426950408889634);
  p.status = a.status;
  const uint64_t bt = static_cast<uint64_t>(a.B) * a.T;
  auto map = [&](const void* base, int H) {
    return make_tmap_3d_bf16(base, fab::kD, H, bt, fab::kD, static_cast<uint64_t>(H) * fab::kD, 64, 1, 128, true);
  };
  const CUtensorMap tq = map(a.q, a.Hq), tk = map(a.k, a.Hkv), tv = map(a.v, a.Hkv), tdo = map(a.dout, a.Hq);
  const CUtensorMap tdq = dq_acc_map(a.dq_acc, a.B, a.T, a.Hq);
  dim3 grid((a.T + fab::kB - 1) / fab::kB, a.Hkv, a.B);
  fab::fa_bwd_kernel<<<grid, fab::kThreads, flash_attn_bwd_smem_bytes(), stream>>>(tq, tk, tv, tdo, tdq, p);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  const long long n4 = rows * fab::kD / 4;
  fab::fa_cast_kernel<<<static_cast<int>(std::min<long long>((n4 + 255) / 256, 148LL * 16)), 256, 0, stream>>>(
      a.dq_acc, static_cast<__nv_bfloat16*>(a.dq), n4);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

int flash_attn_bwd_smem_bytes() { return static_cast<int>(sizeof(fab::Smem)) + 1024; }

void flash_attn_bwd_configure_current_device() {
  int dev = 0;
  MINT_CUDA_CHECK(cudaGetDevice(&dev));
  check_smem_optin(flash_attn_bwd_smem_bytes(), dev, "fa_bwd_kernel");
  MINT_CUDA_CHECK(cudaFuncSetAttribute(fab::fa_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       flash_attn_bwd_smem_bytes()));
}

}  // namespace mint
