// FlashAttention forward for sm_100a on tcgen05 tensor cores (head_dim 128, bf16, GQA).
//
// One CTA per (128-query tile, query head, batch); 384 threads:
//   warp 0      TMA producer: Q once, then K_j / V_j tiles into 2-stage rings (128B swizzle)
//   warp 1      TMEM owner + single-thread MMA issue:
//                 S_j = Q K_j^T   (M=128 queries, N=128 keys, K=128)  -> TMEM S buffer j%2
//                 O  += P_j V_j   (M=128, N=128 head dims, K=128 keys, P from shared memory)
//               S_{j+1} is issued before PV_j so the softmax of tile j+1 overlaps PV_j.
//   warps 4..   softmax, kSplit per TMEM lane quadrant: each thread owns kCols columns of one
//               query row, loads its scores with tcgen05.ld, applies causal / sliding-window /
//               document / sequence-end masks, exchanges its partial row maximum with the other
//               parts of the row through shared memory (one mbarrier per quadrant), computes
//               P = exp2(s * scale - m) two elements per instruction (packed fp32 FMA, bf16x2 MUFU
//               exponential) with a lazily updated running max (its columns of O are rescaled in
//               TMEM only when the max grows by more than 2^8), writes its part of P (bf16) in the
//               128B-swizzled K-major layout the PV MMA reads, and finally normalizes its columns
//               of O, stores them and the log-sum-exp.
// Tiles outside the causal / window band are never visited. All waits are bounded.
#include <cstdlib>

#include "common.cuh"
#include "host_common.h"

namespace mint {
namespace fa {

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kD = 128;
constexpr int kSplit = 2;                       // softmax warps per TMEM lane quadrant (4 measured slower)
constexpr int kCols = 128 / kSplit;              // score / output columns per softmax thread
constexpr int kThreads = (4 + 4 * kSplit) * 32;  // warp 0 TMA, warp 1 MMA, warps 4.. softmax
constexpr int kTileBytes = kBM * kD * 2;  // 32 KB: one 128 x 128 bf16 tile (two 64-wide swizzle atoms)
constexpr int kAtomBytes = kTileBytes / 2;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct FwdParams {
  __nv_bfloat16* o;       // [B, T, Hq, D]
  float* lse;             // [B, Hq, T]
  const int* doc;         // [B, T] or null
  const int2* dbounds;    // [B, T] document run [start, end) of each token; start < 0: row not sorted
  int B, T, Hq, Hkv;
  int causal, window;     // window < 0: none
  float scale_log2;       // softmax scale * log2(e)
  int diag;               // timing diagnostics (MINT_FA_DIAG bits): 1 exp2 replaced by a multiply-add,
                          // 2 MMAs not issued (results meaningless; for isolating pipeline stages)
  uint32_t* status;
  // MINT_FA_TRACE=1: clock64 stamps of block (0, 0, 0) -- the longest causal query tile -- for the
  // first kTraceTiles key tiles: [softmax half][tile][kTraceSteps] from lane 0 of warps 4 and 8,
  // then [tile][4] from the MMA thread (diagnostics only; null otherwise)
  unsigned long long* trace;
};
constexpr int kTraceTiles = 64;
constexpr int kTraceSteps = 10;

struct Smem {
  uint8_t q[kTileBytes];
  uint8_t k[2][kTileBytes];
  uint8_t v[2][kTileBytes];
  uint8_t p[kTileBytes];
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];
  uint64_t p_full;
  uint64_t pv_done;
  uint64_t mma_done;
  uint64_t mx_full[4];     // per TMEM lane quadrant: every softmax warp of the quadrant published its
                           // partial row maxima (and, last, row sums)
  float mx[2][kSplit][kBM];  // [tile parity][column part][row] partial maxima of the current score tile
  float lsum[kSplit][kBM];   // [column part][row] partial row sums, exchanged once at the end
  uint32_t tmem_base;
  int abort_flag;
};
// dynamic shared memory = the struct + 1024 bytes of alignment slack; 232448 is the per-block opt-in limit
static_assert(sizeof(Smem) + 1024 <= 232448, "shared-memory layout exceeds the per-block limit");


// Key tiles a query tile visits. With sorted document ids, keys before the document of the tile's
// first query and (non-causal) after the document of its last query are skipped.
__device__ __forceinline__ void kv_range(int q0, int T, int causal, int window, const int2* db, int& j0, int& j1) {
  const int q_last = min(T, q0 + kBM) - 1;
  int hi = causal ? q_last + 1 : T;
  int lo = window >= 0 ? max(0, q0 - window) : 0;
  if (db != nullptr) {
    const int2 f = db[q0], l = db[q_last];
    if (f.x >= 0) {
      lo = max(lo, f.x);
      hi = min(hi, l.y);
    }
  }
  j0 = lo / kBN;
  j1 = max(j0, (hi + kBN - 1) / kBN);
}

// S = Q K^T: both operands K-major (head dim contiguous), 2 swizzle atoms along K.
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_addr, uint32_t k_addr) {
  constexpr uint32_t idesc = umma_idesc_bf16(kBM, kBN, false, false);
#pragma unroll
  for (int k = 0; k < kD / 16; ++k) {
    const uint32_t off = (k >> 2) * kAtomBytes + (k & 3) * 32;
    umma_bf16(d_tmem, umma_desc_sw128(q_addr + off, 16, 1024), umma_desc_sw128(k_addr + off, 16, 1024), idesc,
              k > 0 ? 1u : 0u);
  }
}

// O += P V: P K-major (keys contiguous, 2 atoms along K); V MN-major (head dim contiguous):
// atoms of 64 head dims x 128 key rows (16 KB apart), 16 keys = 2048 bytes per K step.
__device__ __forceinline__ void issue_pv(uint32_t d_tmem, uint32_t p_addr, uint32_t v_addr, bool accumulate) {
  constexpr uint32_t idesc = umma_idesc_bf16(kBM, kD, false, true);
#pragma unroll
  for (int k = 0; k < kBN / 16; ++k) {
    const uint32_t poff = (k >> 2) * kAtomBytes + (k & 3) * 32;
    umma_bf16(d_tmem, umma_desc_sw128(p_addr + poff, 16, 1024), umma_desc_sw128(v_addr + k * 2048, kAtomBytes, 1024),
              idesc, (accumulate || k > 0) ? 1u : 0u);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap to, FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hkv);
  const int q0 = qt * kBM;
  const int2* db = p.dbounds != nullptr ? p.dbounds + static_cast<long long>(b) * p.T : nullptr;
  int j0, j1;
  kv_range(q0, p.T, p.causal, p.window, db, j0, j1);
  const int n = j1 - j0;
  volatile int* abort_flag = &s.abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
      mbar_init(&s.s_full[i], 1);
    }
    mbar_init(&s.p_full, 4 * kSplit);
    for (int i = 0; i < 4; ++i) mbar_init(&s.mx_full[i], kSplit);
    mbar_init(&s.pv_done, 1);
    mbar_init(&s.mma_done, 1);
    s.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&s.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  const uint32_t tmem_o = tmem + 256;

  if (warp == 0) {
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      const int qrow = b * p.T + q0;
      mbar_arrive_expect_tx(&s.q_full, kTileBytes);
      tma_load_3d(s.q, &tq, &s.q_full, 0, h, qrow);
      tma_load_3d(s.q + kAtomBytes, &tq, &s.q_full, 64, h, qrow);
      for (int t = 0; t < n; ++t) {
        const int st = t & 1;
        const uint32_t ph = (t >> 1) & 1;
        const int krow = b * p.T + (j0 + t) * kBN;
        if (!mbar_wait(&s.k_empty[st], ph ^ 1u, p.status, kStatusTimeoutAttention, abort_flag)) break;
        mbar_arrive_expect_tx(&s.k_full[st], kTileBytes);
        tma_load_3d(s.k[st], &tk, &s.k_full[st], 0, hk, krow);
        tma_load_3d(s.k[st] + kAtomBytes, &tk, &s.k_full[st], 64, hk, krow);
        if (!mbar_wait(&s.v_empty[st], ph ^ 1u, p.status, kStatusTimeoutAttention, abort_flag)) break;
        mbar_arrive_expect_tx(&s.v_full[st], kTileBytes);
        tma_load_3d(s.v[st], &tv, &s.v_full[st], 0, hk, krow);
        tma_load_3d(s.v[st] + kAtomBytes, &tv, &s.v_full[st], 64, hk, krow);
      }
      if (*abort_flag) {
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n > 0) {
      const uint32_t q_addr = smem_u32(s.q);
      const uint32_t p_addr = smem_u32(s.p);
      bool ok = mbar_wait(&s.q_full, 0, p.status, kStatusTimeoutAttention, abort_flag);
      if (ok && (ok = mbar_wait(&s.k_full[0], 0, p.status, kStatusTimeoutAttention, abort_flag))) {
        tc_fence_after();
        if (!(p.diag & 2)) issue_qk(tmem, q_addr, smem_u32(s.k[0]));
        umma_commit(&s.s_full[0]);
        umma_commit(&s.k_empty[0]);
      }
      unsigned long long* tr = (p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
                                   ? p.trace + 2 * kTraceTiles * kTraceSteps
                                   : nullptr;
      for (int t = 0; t < n && ok; ++t) {
        if (tr != nullptr && t < kTraceTiles) tr[t * 4] = clock64();
        if (t + 1 < n) {
          const int st = (t + 1) & 1;
          if (!mbar_wait(&s.k_full[st], ((t + 1) >> 1) & 1, p.status, kStatusTimeoutAttention, abort_flag)) break;
          tc_fence_after();
          if (!(p.diag & 2)) issue_qk(tmem + st * 128, q_addr, smem_u32(s.k[st]));
          umma_commit(&s.s_full[st]);
          umma_commit(&s.k_empty[st]);
        }
        if (tr != nullptr && t < kTraceTiles) tr[t * 4 + 1] = clock64();
        if (!mbar_wait(&s.p_full, t & 1, p.status, kStatusTimeoutAttention, abort_flag)) break;
        if (tr != nullptr && t < kTraceTiles) tr[t * 4 + 2] = clock64();
        if (!mbar_wait(&s.v_full[t & 1], (t >> 1) & 1, p.status, kStatusTimeoutAttention, abort_flag)) break;
        tc_fence_after();
        if (!(p.diag & 2)) issue_pv(tmem_o, p_addr, smem_u32(s.v[t & 1]), t > 0);
        if (tr != nullptr && t < kTraceTiles) tr[t * 4 + 3] = clock64();
        umma_commit(&s.pv_done);
        umma_commit(&s.v_empty[t & 1]);
      }
      umma_commit(&s.mma_done);
      mbar_wait(&s.mma_done, 0, p.status, kStatusTimeoutAttention, nullptr);
    }
  } else if (warp >= 4) {
    // warp 4 + 4 part + q: TMEM lane quadrant q (query rows q*32 .. q*32+31), score / O columns
    // [kCols part, kCols part + kCols)
    const int q = warp & 3;
    const int part = (warp - 4) >> 2;
    const int cb = part * kCols;
    const int r = q * 32 + lane;
    const int qi = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int doc_q = (p.doc != nullptr && qi < p.T) ? p.doc[static_cast<long long>(b) * p.T + qi] : 0;
    // doc_sorted: document masks come from the bounds; else ids (if given) are compared per element
    const bool doc_sorted = db != nullptr && db[q0].x >= 0;
    const int2 dq = (doc_sorted && qi < p.T) ? db[qi] : make_int2(0, p.T);
    const int d_lo = dq.x, d_hi = dq.y;
    // the tile's keys lie inside every row's document when the last row's document starts before
    // the first key and the first row's document ends after the last key
    const int2 dfirst = doc_sorted ? db[q0] : make_int2(0, p.T);
    const int2 dlast = doc_sorted ? db[min(p.T, q0 + kBM) - 1] : make_int2(0, p.T);
    float m = -INFINITY, l = 0.f;  // running max (shared by every part of the row), this part's row sum
    bool ok = n > 0;
    int pv_waited = -1;  // index of the last PV whose completion this thread observed
    unsigned long long* tr = (p.trace != nullptr && lane == 0 && (warp == 4 || warp == 4 + 4 * (kSplit - 1)) &&
                              blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
                                 ? p.trace + (part == 0 ? 0 : 1) * kTraceTiles * kTraceSteps
                                 : nullptr;
#define FA_STAMP(k) \
  if (tr != nullptr && t < kTraceTiles) tr[t * kTraceSteps + (k)] = clock64();
    for (int t = 0; t < n && ok; ++t) {
      const int kb = (j0 + t) * kBN;
      FA_STAMP(0)
      if (!mbar_wait_warp(&s.s_full[t & 1], (t >> 1) & 1, p.status, kStatusTimeoutAttention, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      FA_STAMP(1)
      float x[kCols];  // raw scores: the softmax scale goes into the exponent's FMA
      {
        uint32_t u[kCols];
#pragma unroll
        for (int c = 0; c < kCols / 32; ++c) {
          tmem_ld_32x32b_x32(tmem + (t & 1) * 128 + lane_off + cb + c * 32,
                             *reinterpret_cast<uint32_t(*)[32]>(u + c * 32));
        }
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < kCols; ++e) x[e] = __uint_as_float(u[e]);
      }
      const bool doc_mask = p.doc != nullptr && !(doc_sorted && dlast.x <= kb && dfirst.y >= kb + kBN);
      const bool need_mask = (p.causal && kb + kBN - 1 > q0) || (p.window >= 0 && q0 + kBM - 1 - kb > p.window) ||
                             kb + kBN > p.T || doc_mask;
      if (need_mask) {
        if (doc_sorted || p.doc == nullptr) {
#pragma unroll
          for (int c = 0; c < kCols; ++c) {
            const int kj = kb + cb + c;
            bool keep = kj < p.T && kj >= d_lo && kj < d_hi;
            if (p.causal) keep = keep && kj <= qi;
            if (p.window >= 0) keep = keep && qi - kj <= p.window;
            if (!keep) x[c] = -INFINITY;
          }
        } else {
          for (int c = 0; c < kCols; ++c) {
            const int kj = kb + cb + c;
            bool keep = kj < p.T;
            if (p.causal) keep = keep && kj <= qi;
            if (p.window >= 0) keep = keep && qi - kj <= p.window;
            if (keep) keep = p.doc[static_cast<long long>(b) * p.T + kj] == doc_q;
            if (!keep) x[c] = -INFINITY;
          }
        }
      }
      FA_STAMP(2)
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // four independent chains
#pragma unroll
      for (int c = 0; c < kCols; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], x[c]);
      float mt = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      FA_STAMP(3)
      // combine with the other parts of the row; the buffer of this parity was last read two tiles
      // ago, before every warp of the quadrant arrived on the previous tile's exchange
      s.mx[t & 1][part][r] = mt;
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.mx_full[q]);
      if (!mbar_wait_warp(&s.mx_full[q], t & 1, p.status, kStatusTimeoutAttention, abort_flag)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int o2 = 0; o2 < kSplit; ++o2) {
        if (o2 != part) mt = fmaxf(mt, s.mx[t & 1][o2][r]);
      }
      FA_STAMP(4)
      const float m_new = fmaxf(m, mt * p.scale_log2);  // running max in scaled log2 units
      // tcgen05.ld/st are warp-collective: the rescale decision must be uniform across the warp; the
      // warps of a lane quadrant see the same row maxima and so decide alike
      const bool grow = m != -INFINITY && m_new > m + kRescaleThreshold;
      if (t > 0 && __any_sync(0xffffffffu, grow)) {
        // O holds PV_0..PV_{t-1}: wait for PV_{t-1}, then rescale this part of the rows in TMEM
        if (pv_waited < t - 1) {
          if (!mbar_wait_warp(&s.pv_done, (t - 1) & 1, p.status, kStatusTimeoutAttention, abort_flag)) {
            ok = false;
            break;
          }
          pv_waited = t - 1;
          tc_fence_after();
        }
        const float alpha = (m == -INFINITY || m_new == -INFINITY) ? 0.f : exp2f(m - m_new);
        l *= alpha;
#pragma unroll
        for (int c = 0; c < kCols / 16; ++c) {
          uint32_t u[16];
          tmem_ld_32x32b_x16(tmem_o + lane_off + cb + c * 16, u);
          tmem_ld_wait();
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) w[e] = __float_as_uint(__uint_as_float(u[e]) * alpha);
          tmem_st_32x32b_x16(tmem_o + lane_off + cb + c * 16, w);
        }
        tmem_st_wait();
        m = m_new;
      } else if (m == -INFINITY) {
        m = m_new;  // nothing accumulated in this row yet
      }
      FA_STAMP(5)
      // P = exp2(x * scale - m) in bf16, two elements per instruction (packed fp32 FMA, bf16x2 MUFU
      // exponential); the row sum adds the bf16 values the PV MMA uses. A row with nothing kept yet
      // (m = -inf) has every x = -inf, so m is taken as 0 there and every p comes out 0.
      uint32_t pk[kCols / 2];
      float rs = 0.f;
      {
        const float mm = (m == -INFINITY) ? 0.f : m;
        const float2 sc2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(-mm, -mm);
        float2 acc2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};  // two chains for ILP
#pragma unroll
        for (int c = 0; c < kCols / 2; ++c) {
          const float2 tt = ffma2(make_float2(x[2 * c], x[2 * c + 1]), sc2, nm2);
          uint32_t e;
          if (p.diag & 1) {
            e = pack_bf16x2(fmaf(tt.x, 0.01f, 1.f), fmaf(tt.y, 0.01f, 1.f));
          } else {
            e = ex2_bf16x2(tt.x, tt.y);
          }
          pk[c] = e;
          acc2[c & 1] = fadd2(acc2[c & 1], bf16x2_to_float2(e));
        }
        rs = (acc2[0].x + acc2[1].x) + (acc2[0].y + acc2[1].y);
      }
      l += rs;
      FA_STAMP(6)
      // the single P buffer is free once PV_{t-1} completed
      if (t > 0 && pv_waited < t - 1) {
        if (!mbar_wait_warp(&s.pv_done, (t - 1) & 1, p.status, kStatusTimeoutAttention, abort_flag)) {
          ok = false;
          break;
        }
        pv_waited = t - 1;
      }
      FA_STAMP(7)
      // 128B-swizzled K-major store of this part of the row: 64-key swizzle atom cb / 64, 16-byte
      // chunk (cb % 64) / 8 + c at that index ^ (row % 8)
#pragma unroll
      for (int c = 0; c < kCols / 8; ++c) {
        const int chunk = (cb & 63) / 8 + c;
        const uint4 v4 = make_uint4(pk[c * 4], pk[c * 4 + 1], pk[c * 4 + 2], pk[c * 4 + 3]);
        *reinterpret_cast<uint4*>(s.p + (cb >> 6) * kAtomBytes + r * 128 + ((chunk ^ (r & 7)) << 4)) = v4;
      }
      FA_STAMP(8)
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.p_full);
      FA_STAMP(9)
    }
#undef FA_STAMP
    if (ok && n > 0 && pv_waited < n - 1) {
      ok = mbar_wait_warp(&s.pv_done, (n - 1) & 1, p.status, kStatusTimeoutAttention, abort_flag);
    }
    // row sum over every part (a final exchange round on mx_full, phase n)
    if (ok && n > 0) {
      s.lsum[part][r] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.mx_full[q]);
      ok = mbar_wait_warp(&s.mx_full[q], n & 1, p.status, kStatusTimeoutAttention, abort_flag);
      if (ok) {
        l = 0.f;
#pragma unroll
        for (int o2 = 0; o2 < kSplit; ++o2) l += s.lsum[o2][r];
      }
    }
    ok = __all_sync(0xffffffffu, ok);
    if (ok && n > 0) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool row_ok = qi < p.T;
      // each thread stores its row's kCols output columns directly (rows past the sequence end skip)
      __nv_bfloat16* orow = p.o + ((static_cast<long long>(b) * p.T + (row_ok ? qi : 0)) * p.Hq + h) * kD + cb;
#pragma unroll
      for (int c = 0; c < kCols / 32; ++c) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(tmem_o + lane_off + cb + c * 32, u);  // warp-collective: every lane loads
        tmem_ld_wait();
        if (!row_ok) continue;
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 v4;
          v4.x = pack_bf16x2(__uint_as_float(u[e]) * inv, __uint_as_float(u[e + 1]) * inv);
          v4.y = pack_bf16x2(__uint_as_float(u[e + 2]) * inv, __uint_as_float(u[e + 3]) * inv);
          v4.z = pack_bf16x2(__uint_as_float(u[e + 4]) * inv, __uint_as_float(u[e + 5]) * inv);
          v4.w = pack_bf16x2(__uint_as_float(u[e + 6]) * inv, __uint_as_float(u[e + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c * 32 + e) = v4;
        }
      }
      // natural-log LSE of the scaled scores: (m + log2 l) * ln 2
      if (row_ok && part == 0) {
        p.lse[(static_cast<long long>(b) * p.Hq + h) * p.T + qi] =
            l > 0.f ? (m + log2f(l)) * 0.6931471805599453f : -INFINITY;
      }
    } else if (n == 0 && qi < p.T) {
      __nv_bfloat16* orow = p.o + ((static_cast<long long>(b) * p.T + qi) * p.Hq + h) * kD + cb;
      for (int c = 0; c < kCols; ++c) orow[c] = __float2bfloat16_rn(0.f);
      if (part == 0) p.lse[(static_cast<long long>(b) * p.Hq + h) * p.T + qi] = -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Document run of every token for attention's tile skipping: with the row's ids non-decreasing,
// token t's document is [lower_bound(doc[t]), upper_bound(doc[t])) of the row (binary searches).
// Rows whose ids ever decrease get start = end = -1 (kernels then compare ids and skip nothing).
__global__ void __launch_bounds__(256) doc_bounds_kernel(const int* __restrict__ doc, int2* __restrict__ out, int T) {
  const int b = blockIdx.x;
  const int* row = doc + static_cast<long long>(b) * T;
  int unsorted = 0;
  for (int t = threadIdx.x + 1; t < T; t += blockDim.x) unsorted |= row[t] < row[t - 1];
  unsorted = __syncthreads_or(unsorted);
  int2* o = out + static_cast<long long>(b) * T;
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    if (unsorted) {
      o[t] = make_int2(-1, -1);
      continue;
    }
    const int v = row[t];
    int lo = 0, hi = t;  // first index with row[i] >= v lies in [0, t]
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (row[mid] < v) lo = mid + 1; else hi = mid;
    }
    int lo2 = t + 1, hi2 = T;  // first index with row[i] > v lies in [t + 1, T]
    while (lo2 < hi2) {
      const int mid = (lo2 + hi2) >> 1;
      if (row[mid] <= v) lo2 = mid + 1; else hi2 = mid;
    }
    o[t] = make_int2(lo, lo2);
  }
}

}  // namespace fa

at::Tensor doc_bounds(const at::Tensor& doc) {
  check_contig(doc, "doc_ids");
  MINT_CHECK(doc.scalar_type() == at::kInt && doc.dim() == 2, "doc_ids must be int32 [B, T]");
  const int B = static_cast<int>(doc.size(0)), T = static_cast<int>(doc.size(1));
  auto out = at::empty({B, T, 2}, doc.options());
  if (B == 0 || T == 0) return out;
  c10::cuda::CUDAGuard guard(doc.device());
  fa::doc_bounds_kernel<<<B, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      doc.data_ptr<int>(), reinterpret_cast<int2*>(out.data_ptr<int>()), T);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return out;
}

const int2* doc_bounds_ptr(const c10::optional<at::Tensor>& doc, const c10::optional<at::Tensor>& dbounds,
                           int64_t B, int64_t T, at::Tensor& holder) {
  if (!doc.has_value() || !doc->defined()) return nullptr;
  if (dbounds.has_value() && dbounds->defined()) {
    check_contig(*dbounds, "doc bounds");
    MINT_CHECK(dbounds->scalar_type() == at::kInt && dbounds->numel() == 2 * B * T, "doc bounds must be int32 [B, T, 2]");
    holder = *dbounds;
  } else {
    holder = doc_bounds(doc->view({B, T}));
  }
  return reinterpret_cast<const int2*>(holder.data_ptr<int>());
}

// MINT_FA_TRACE=1 diagnostics: the stamp buffer of the last forward (zeros if tracing is off)
at::Tensor& fa_trace_buffer() {
  static at::Tensor buf;
  return buf;
}

at::Tensor flash_attn_fwd_trace() {
  at::Tensor& buf = fa_trace_buffer();
  return buf.defined() ? buf.clone() : at::zeros({(2 * fa::kTraceSteps + 4) * fa::kTraceTiles}, at::kLong);
}

std::vector<at::Tensor> flash_attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                       const c10::optional<at::Tensor>& doc, bool causal, int64_t window,
                                       double scale, const c10::optional<at::Tensor>& dbounds) {
  check_contig(q, "q");
  check_contig(k, "k");
  check_contig(v, "v");
  MINT_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
             "flash_attn expects bf16");
  MINT_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "flash_attn expects [B, T, H, D]");
  const int B = static_cast<int>(q.size(0)), T = static_cast<int>(q.size(1));
  const int Hq = static_cast<int>(q.size(2)), Hkv = static_cast<int>(k.size(2));
  MINT_CHECK(q.size(3) == fa::kD && k.size(3) == fa::kD && v.size(3) == fa::kD, "head_dim must be 128");
  MINT_CHECK(k.size(1) == T && v.size(1) == T && k.size(0) == B && v.sizes() == k.sizes(), "k/v shape mismatch");
  MINT_CHECK(Hq % Hkv == 0, "Hq must be a multiple of Hkv");
  auto o = at::empty_like(q);
  auto lse = at::empty({B, Hq, T}, q.options().dtype(at::kFloat));
  if (B == 0 || T == 0) return {o, lse};
  c10::cuda::CUDAGuard guard(q.device());
  fa::FwdParams p{};
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.lse = lse.data_ptr<float>();
  if (doc.has_value() && doc->defined()) {
    check_contig(*doc, "doc_ids");
    MINT_CHECK(doc->scalar_type() == at::kInt && doc->numel() == static_cast<int64_t>(B) * T, "doc_ids must be int32 [B, T]");
    p.doc = doc->data_ptr<int>();
  }
  at::Tensor bounds_holder;
  p.dbounds = doc_bounds_ptr(doc, dbounds, B, T, bounds_holder);
  p.B = B;
  p.T = T;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.causal = causal ? 1 : 0;
  p.window = static_cast<int>(window);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.status = status_ptr(q.get_device());
  static const int diag = [] {
    const char* e = std::getenv("MINT_FA_DIAG");
    return e == nullptr ? 0 : std::atoi(e);
  }();
  p.diag = diag;
  static const bool trace = std::getenv("MINT_FA_TRACE") != nullptr;
  if (trace) {
    at::Tensor& buf = fa_trace_buffer();
    if (!buf.defined() || buf.device() != q.device()) {
      buf = at::zeros({(2 * fa::kTraceSteps + 4) * fa::kTraceTiles}, q.options().dtype(at::kLong));
    }
    p.trace = reinterpret_cast<unsigned long long*>(buf.data_ptr<int64_t>());
  }
  const CUtensorMap tq = make_tmap_3d_bf16(q.data_ptr(), fa::kD, Hq, static_cast<uint64_t>(B) * T, fa::kD,
                                           static_cast<uint64_t>(Hq) * fa::kD, 64, 1, 128, true);
  const CUtensorMap tk = make_tmap_3d_bf16(k.data_ptr(), fa::kD, Hkv, static_cast<uint64_t>(B) * T, fa::kD,
                                           static_cast<uint64_t>(Hkv) * fa::kD, 64, 1, 128, true);
  const CUtensorMap tv = make_tmap_3d_bf16(v.data_ptr(), fa::kD, Hkv, static_cast<uint64_t>(B) * T, fa::kD,
                                           static_cast<uint64_t>(Hkv) * fa::kD, 64, 1, 128, true);
  const int smem = static_cast<int>(sizeof(fa::Smem)) + 1024;
  static bool configured[64] = {};  // the attribute is per device
  const int dev = q.get_device();
  auto kern = fa::fa_fwd_kernel;
  if (!configured[dev & 63]) {
    check_smem_optin(smem, dev, "fa_fwd_kernel");
    MINT_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured[dev & 63] = true;
  }
  dim3 grid((T + fa::kBM - 1) / fa::kBM, Hq, B);
  // O leaves in 32-row x 64-dim boxes, one TMA store per softmax warp
  const CUtensorMap to = make_tmap_3d_bf16(o.data_ptr(), fa::kD, Hq, static_cast<uint64_t>(B) * T, fa::kD,
                                           static_cast<uint64_t>(Hq) * fa::kD, 64, 1, 32, true);
  kern<<<grid, fa::kThreads, smem, at::cuda::getCurrentCUDAStream()>>>(tq, tk, tv, to, p);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return {o, lse};
}

}  // namespace mint
