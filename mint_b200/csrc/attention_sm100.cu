// FlashAttention forward for sm_100a on tcgen05 tensor cores (head_dim 128, bf16, GQA).
//
// One CTA per (256 queries, query head, batch): two 128-row query tiles X = 0, 1 that share every
// K / V tile the TMA warp streams in. Tensor memory holds, per tile, S_X (128 fp32 columns) and O_X
// (128 fp32 columns): all 512 columns. 320 threads:
//   warp 0      TMA producer: Q_0, Q_1 once, then K_j / V_j into 2-stage rings (128B swizzle)
//   warp 1      TMEM owner + single-thread MMA issue, ping-ponging the tiles:
//                 S_X(j) = Q_X K_j^T  (SMEM x SMEM -> TMEM)
//                 O_X   += P_X(j) V_j (P read from TMEM, V from SMEM)
//               after issuing PV_X(j) it waits for it and issues S_X(j+1) into the same columns,
//               so one tile's softmax runs while the tensor pipe works on the other tile
//   warps 2..5  softmax of tile 0, warps 6..9 softmax of tile 1: one thread per query row (warp w
//               owns TMEM lane quadrant w % 4), the whole 128-key row in registers -- no cross-warp
//               exchange. Masks (causal / sliding window / document / sequence end), row max, a
//               lazy O rescale in TMEM (only when the max grows by more than 2^8), exp2 (a quarter
//               of them on the FMA pipe, exp2_poly), P packed to bf16 and written back over the
//               first 64 columns of S_X for the PV MMA; at the end O / l leaves through shared
//               memory (the tile's Q buffer) with one TMA store per warp and 64 columns, and the
//               natural-log LSE is stored per row.
// Key tiles outside a query tile's causal / window / document band are skipped per tile. Every
// wait is bounded; on a timeout the kernel records a status bit, drains and returns.
#include <cstdlib>

#include "common.cuh"
#include "host_common.h"

namespace mint {
namespace fa {

constexpr int kBM = 128;       // query rows per tile
constexpr int kTiles = 2;      // query tiles per CTA
constexpr int kBN = 128;       // keys per K / V tile
constexpr int kD = 128;
constexpr int kStages = 2;
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2..5 / 6..9 softmax of tile 0 / 1 (~200 registers each)
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
  uint32_t* status;
};

struct Smem {
  uint8_t q[kTiles][kTileBytes];  // reused as the O staging buffer of the tile at the end
  uint8_t k[kStages][kTileBytes];
  uint8_t v[kStages][kTileBytes];
  uint64_t q_full;
  uint64_t k_full[kStages], k_empty[kStages];
  uint64_t v_full[kStages], v_empty[kStages];
  uint64_t s_full[kTiles];   // S_X(j) in TMEM (MMA commit)
  uint64_t p_full[kTiles];   // P_X(j) written over S_X (4 softmax warps)
  uint64_t pv_done[kTiles];  // PV_X(j) complete (MMA commit)
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};
// dynamic shared memory = the struct + 1024 bytes of alignment slack; 232448 is the per-block opt-in limit
static_assert(sizeof(Smem) + 1024 <= 232448, "shared-memory layout exceeds the per-block limit");

// Key tiles a query tile visits. With sorted document ids, keys before the document of the tile's
// first query and (non-causal) after the document of its last query are skipped.
__device__ __forceinline__ void kv_range(int q0, int T, int causal, int window, const int2* db, int& j0, int& j1) {
  if (q0 >= T) {
    j0 = j1 = 0;
    return;
  }
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

// O += P V with P (bf16, two per 32-bit column, keys along columns) read from tensor memory and V
// MN-major from shared memory (atoms of 64 head dims x 128 key rows, 16 KB apart; 16 keys = 2048 B).
__device__ __forceinline__ void issue_pv_tmem(uint32_t o_tmem, uint32_t p_tmem, uint32_t v_addr, bool accumulate) {
  constexpr uint32_t idesc = umma_idesc_bf16(kBM, kD, false, true);
#pragma unroll
  for (int k = 0; k < kBN / 16; ++k) {
    umma_bf16_tmem_a(o_tmem, p_tmem + k * 8, umma_desc_sw128(v_addr + k * 2048, kAtomBytes, 1024), idesc,
                     (accumulate || k > 0) ? 1u : 0u);
  }
}

// Which keys one query row keeps in the current key tile.
struct RowMask {
  bool need, by_range;
  int lo, hi, qi, T, causal, window, doc_q;
  const int* doc_row;
  __device__ __forceinline__ bool keep(int kj) const {
    if (!need) return true;
    if (by_range) return kj >= lo && kj < hi;
    const bool k = kj < T && (!causal || kj <= qi) && (window < 0 || qi - kj <= window);
    return k && doc_row[kj] == doc_q;
  }
};

// Bit e set when key base + e (e < 32) is kept by row mask `mk`: arithmetic for a [lo, hi) range,
// one id comparison per key (not unrolled) for unsorted document ids.
__device__ __forceinline__ uint32_t chunk_keep_mask(const RowMask& mk, int base) {
  if (!mk.need) return 0xffffffffu;
  if (mk.by_range) {
    const int a = max(mk.lo - base, 0), z = min(mk.hi - base, 32);
    if (a >= z) return 0u;
    const uint32_t upto = z >= 32 ? 0xffffffffu : ((1u << z) - 1u);
    return upto & ~((1u << a) - 1u);
  }
  uint32_t bits = 0u;
#pragma unroll 1
  for (int e = 0; e < 32; ++e) bits |= (mk.keep(base + e) ? 1u : 0u) << e;
  return bits;
}

// Key-tile ranges [j0, j1) of the CTA's two query tiles, held in scalars (no per-thread local array)
struct TileRanges {
  int a0, a1, b0, b1;
  __device__ __forceinline__ int lo(int x) const { return x ? b0 : a0; }
  __device__ __forceinline__ int hi(int x) const { return x ? b1 : a1; }
  __device__ __forceinline__ bool active(int x, int j) const { return j >= lo(x) && j < hi(x); }
};

// 320 threads, one CTA per SM: a 200-register budget per thread (instead of a launch bound, which
// made ptxas settle at 168 and spill the 128 scores each softmax thread holds)
__global__ void __maxnreg__(200)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap to, FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = gridDim.x - 1 - blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hkv);
  const int q0 = qb * (kTiles * kBM);
  const int2* db = p.dbounds != nullptr ? p.dbounds + static_cast<long long>(b) * p.T : nullptr;
  TileRanges tr;
  kv_range(q0, p.T, p.causal, p.window, db, tr.a0, tr.a1);
  kv_range(q0 + kBM, p.T, p.causal, p.window, db, tr.b0, tr.b1);
  int u0 = 1 << 30, u1 = 0;  // union of the tiles' key ranges
#pragma unroll
  for (int x = 0; x < kTiles; ++x) {
    if (tr.hi(x) > tr.lo(x)) {
      u0 = min(u0, tr.lo(x));
      u1 = max(u1, tr.hi(x));
    }
  }
  const int n = u1 > u0 ? u1 - u0 : 0;
  volatile int* abort_flag = &s.abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
    }
    for (int x = 0; x < kTiles; ++x) {
      mbar_init(&s.s_full[x], 1);
      mbar_init(&s.p_full[x], 4);
      mbar_init(&s.pv_done[x], 1);
    }
    mbar_init(&s.mma_done, 1);
    s.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&s.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0) {
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      const int qrow = b * p.T + q0;
      mbar_arrive_expect_tx(&s.q_full, kTiles * kTileBytes);
      for (int x = 0; x < kTiles; ++x) {
        tma_load_3d(s.q[x], &tq, &s.q_full, 0, h, qrow + x * kBM);
        tma_load_3d(s.q[x] + kAtomBytes, &tq, &s.q_full, 64, h, qrow + x * kBM);
      }
      for (int t = 0; t < n; ++t) {
        const int st = t & 1;
        const uint32_t ph = (t >> 1) & 1;
        const int krow = b * p.T + (u0 + t) * kBN;
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
      uint32_t cnt0 = 0, cnt1 = 0;  // PVs issued per tile
      bool ok = mbar_wait(&s.q_full, 0, p.status, kStatusTimeoutAttention, abort_flag);
      if (ok) ok = mbar_wait(&s.k_full[0], 0, p.status, kStatusTimeoutAttention, abort_flag);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int x = 0; x < kTiles; ++x) {
          if (!tr.active(x, u0)) continue;
          issue_qk(tmem + x * 256, smem_u32(s.q[x]), smem_u32(s.k[0]));
          umma_commit(&s.s_full[x]);
        }
        umma_commit(&s.k_empty[0]);
      }
      for (int t = 0; t < n && ok; ++t) {
        const int j = u0 + t;
        const int st = t & 1;
        bool v_ready = false, k_next_ready = false;
#pragma unroll
        for (int x = 0; x < kTiles; ++x) {
          if (!ok || !tr.active(x, j)) continue;
          const uint32_t cnt = x ? cnt1 : cnt0;  // PVs of this tile issued so far
          if (!(ok = mbar_wait(&s.p_full[x], cnt & 1, p.status, kStatusTimeoutAttention, abort_flag))) continue;
          if (!v_ready) {
            if (!(ok = mbar_wait(&s.v_full[st], (t >> 1) & 1, p.status, kStatusTimeoutAttention, abort_flag))) continue;
            v_ready = true;
          }
          tc_fence_after();
          issue_pv_tmem(tmem + x * 256 + 128, tmem + x * 256, smem_u32(s.v[st]), cnt > 0);
          umma_commit(&s.pv_done[x]);
          if (x) ++cnt1; else ++cnt0;
          if (t + 1 < n && tr.active(x, j + 1)) {
            // the next S of this tile overwrites P: wait until the PV just issued has read it
            if (!k_next_ready) {
              if (!(ok = mbar_wait(&s.k_full[(t + 1) & 1], ((t + 1) >> 1) & 1, p.status, kStatusTimeoutAttention,
                                   abort_flag)))
                continue;
              k_next_ready = true;
            }
            if (!(ok = mbar_wait(&s.pv_done[x], cnt & 1, p.status, kStatusTimeoutAttention, abort_flag)))
              continue;
            tc_fence_after();
            issue_qk(tmem + x * 256, smem_u32(s.q[x]), smem_u32(s.k[(t + 1) & 1]));
            umma_commit(&s.s_full[x]);
          }
        }
        if (!ok) break;
        // a step no tile uses still consumed a K / V load: release the slots only after it landed
        if (!v_ready && !(ok = mbar_wait(&s.v_full[st], (t >> 1) & 1, p.status, kStatusTimeoutAttention, abort_flag)))
          break;
        umma_commit(&s.v_empty[st]);
        if (t + 1 < n) {
          // tiles whose first key tile is j + 1 start here
#pragma unroll
          for (int x = 0; x < kTiles; ++x) {
            if (!ok || tr.active(x, j) || !tr.active(x, j + 1)) continue;
            if (!k_next_ready) {
              if (!(ok = mbar_wait(&s.k_full[(t + 1) & 1], ((t + 1) >> 1) & 1, p.status, kStatusTimeoutAttention,
                                   abort_flag)))
                continue;
              k_next_ready = true;
            }
            tc_fence_after();
            issue_qk(tmem + x * 256, smem_u32(s.q[x]), smem_u32(s.k[(t + 1) & 1]));
            umma_commit(&s.s_full[x]);
          }
          if (ok && !k_next_ready) {
            ok = mbar_wait(&s.k_full[(t + 1) & 1], ((t + 1) >> 1) & 1, p.status, kStatusTimeoutAttention, abort_flag);
          }
          if (!ok) break;
          umma_commit(&s.k_empty[(t + 1) & 1]);
        }
      }
      umma_commit(&s.mma_done);
      mbar_wait(&s.mma_done, 0, p.status, kStatusTimeoutAttention, nullptr);
    }
  } else {
    const int x = (warp - 2) >> 2;  // query tile of this warp group
    const int q = warp & 3;         // TMEM lane quadrant (warp % 4): rows q*32 .. q*32+31 of the tile
    const int r = q * 32 + lane;
    const int qt0 = q0 + x * kBM;
    const int qi = qt0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t tmem_s = tmem + x * 256 + lane_off;
    const uint32_t tmem_o = tmem_s + 128;
    const int doc_q = (p.doc != nullptr && qi < p.T) ? p.doc[static_cast<long long>(b) * p.T + qi] : 0;
    // doc_sorted: document masks come from the bounds; else ids (if given) are compared per element
    const bool doc_sorted = db != nullptr && qt0 < p.T && db[qt0].x >= 0;
    const int2 dq = (doc_sorted && qi < p.T) ? db[qi] : make_int2(0, p.T);
    // the tile's keys lie inside every row's document when the last row's document starts before
    // the first key and the first row's document ends after the last key
    const int2 dfirst = doc_sorted ? db[qt0] : make_int2(0, p.T);
    const int2 dlast = doc_sorted ? db[min(p.T, qt0 + kBM) - 1] : make_int2(0, p.T);
    const int jx0 = tr.lo(x);
    const int nx = tr.hi(x) - jx0;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int c = 0; c < nx && ok; ++c) {
      const int kb = (jx0 + c) * kBN;
      if (!mbar_wait_warp(&s.s_full[x], c & 1, p.status, kStatusTimeoutAttention, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool doc_mask = p.doc != nullptr && !(doc_sorted && dlast.x <= kb && dfirst.y >= kb + kBN);
      const bool need_mask = (p.causal && kb + kBN - 1 > qt0) || (p.window >= 0 && qt0 + kBM - 1 - kb > p.window) ||
                             kb + kBN > p.T || doc_mask;
      // kept keys of this row: [lo, hi) (sorted or no document ids), else ids are compared per key
      RowMask mk;
      mk.need = need_mask;
      mk.by_range = doc_sorted || p.doc == nullptr;
      mk.lo = max(dq.x, p.window >= 0 ? qi - p.window : 0);
      mk.hi = min(min(dq.y, p.T), p.causal ? qi + 1 : p.T);
      mk.qi = qi;
      mk.T = p.T;
      mk.causal = p.causal;
      mk.window = p.window;
      mk.doc_q = doc_q;
      mk.doc_row = p.doc != nullptr ? p.doc + static_cast<long long>(b) * p.T : nullptr;
      // the 128 scores of this row: four loads, one wait
      uint32_t u[128];
#pragma unroll
      for (int g = 0; g < 4; ++g) tmem_ld_32x32b_x32(tmem_s + g * 32, *reinterpret_cast<uint32_t(*)[32]>(&u[g * 32]));
      uint32_t kbits[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) kbits[g] = chunk_keep_mask(mk, kb + g * 32);
      tmem_ld_wait();
      float mt = -INFINITY;
#pragma unroll
      for (int e = 0; e < 128; ++e) {
        if ((kbits[e >> 5] >> (e & 31)) & 1u) mt = fmaxf(mt, __uint_as_float(u[e]) * p.scale_log2);
      }
      const float m_new = fmaxf(m, mt);
      // tcgen05.ld / st are warp-collective: the rescale decision is made uniform across the warp
      const bool grow = m != -INFINITY && m_new > m + kRescaleThreshold;
      const bool rescale = c > 0 && __any_sync(0xffffffffu, grow);
      const float alpha = (!rescale || m == -INFINITY || m_new == -INFINITY) ? 1.f : exp2f(m - m_new);
      if (rescale || m == -INFINITY) m = m_new;
      // P = exp2(s - m) in bf16 (a quarter on the FMA pipe), row sum in fp32, written over the first
      // 64 columns of S (their scores are already in registers)
      float rs = 0.f;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float a = 0.f, bb = 0.f;
          const int i0 = g * 32 + 2 * e;
          if (m != -INFINITY) {
            if ((kbits[g] >> (2 * e)) & 1u) a = exp2f(__uint_as_float(u[i0]) * p.scale_log2 - m);
            if ((kbits[g] >> (2 * e + 1)) & 1u) {
              const float t = __uint_as_float(u[i0 + 1]) * p.scale_log2 - m;
              bb = (e & 1) ? exp2_poly(t) : exp2f(t);
            }
          }
          rs += a + bb;
          pk[e] = pack_bf16x2(a, bb);
        }
        tmem_st_32x32b_x16(tmem_s + g * 16, pk);
      }
      if (rescale) {
        // O holds PV_0..PV_{c-1}; PV_{c-1} completed before S(c) was issued into this tile's columns,
        // and PV_c is issued only after this warp signals P ready below
        l *= alpha;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint32_t w[32];
          tmem_ld_32x32b_x32(tmem_o + g * 32, w);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) w[e] = __float_as_uint(__uint_as_float(w[e]) * alpha);
          tmem_st_32x32b_x32(tmem_o + g * 32, w);
        }
      }
      l += rs;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.p_full[x]);
    }
    if (ok && nx > 0) ok = mbar_wait_warp(&s.pv_done[x], (nx - 1) & 1, p.status, kStatusTimeoutAttention, abort_flag);
    ok = __all_sync(0xffffffffu, ok);
    if (ok && nx > 0) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool row_ok = qi < p.T;
      // warps whose 32 rows all lie inside the sequence store through shared memory (this tile's Q
      // buffer: every MMA reading it completed) and TMA; the ragged last warp stores directly
      const bool via_tma = qt0 + q * 32 + 32 <= p.T;
      __nv_bfloat16* orow = p.o + ((static_cast<long long>(b) * p.T + (row_ok ? qi : 0)) * p.Hq + h) * kD;
      uint8_t* stage = s.q[x];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(tmem_o + g * 32, u);  // warp-collective: every lane loads
        tmem_ld_wait();
        if (!row_ok) continue;
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(u[e]) * inv, __uint_as_float(u[e + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(u[e + 2]) * inv, __uint_as_float(u[e + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(u[e + 4]) * inv, __uint_as_float(u[e + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(u[e + 6]) * inv, __uint_as_float(u[e + 7]) * inv);
          const int col = g * 32 + e;  // head dim of w.x
          if (via_tma) {
            const int atom = col >> 6, chunk = (col & 63) >> 3;  // 64-dim swizzle atom, 16-byte chunk
            *reinterpret_cast<uint4*>(stage + atom * kAtomBytes + r * 128 + ((chunk ^ (r & 7)) << 4)) = w;
          } else {
            *reinterpret_cast<uint4*>(orow + col) = w;
          }
        }
      }
      if (via_tma) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          for (int a = 0; a < 2; ++a) tma_store_3d(&to, stage + a * kAtomBytes + q * 32 * 128, a * 64, h, b * p.T + qt0 + q * 32);
          bulk_commit();
          bulk_wait_read<0>();  // the shared memory must stay valid until the stores have read it
        }
        __syncwarp();
      }
      // natural-log LSE of the scaled scores: (m + log2 l) * ln 2
      if (row_ok) {
        p.lse[(static_cast<long long>(b) * p.Hq + h) * p.T + qi] = l > 0.f ? (m + log2f(l)) * 0.6931471805599453f : -INFINITY;
      }
    } else if (nx == 0 && qi < p.T) {
      __nv_bfloat16* orow = p.o + ((static_cast<long long>(b) * p.T + qi) * p.Hq + h) * kD;
      for (int c = 0; c < kD; ++c) orow[c] = __float2bfloat16_rn(0.f);
      p.lse[(static_cast<long long>(b) * p.Hq + h) * p.T + qi] = -INFINITY;
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
  const CUtensorMap tq = make_tmap_3d_bf16(q.data_ptr(), fa::kD, Hq, static_cast<uint64_t>(B) * T, fa::kD,
                                           static_cast<uint64_t>(Hq) * fa::kD, 64, 1, 128, true);
  const CUtensorMap tk = make_tmap_3d_bf16(k.data_ptr(), fa::kD, Hkv, static_cast<uint64_t>(B) * T, fa::kD,
                                           static_cast<uint64_t>(Hkv) * fa::kD, 64, 1, 128, true);
  const CUtensorMap tv = make_tmap_3d_bf16(v.data_ptr(), fa::kD, Hkv, static_cast<uint64_t>(B) * T, fa::kD,
                                           static_cast<uint64_t>(Hkv) * fa::kD, 64, 1, 128, true);
  const int smem = static_cast<int>(sizeof(fa::Smem)) + 1024;
  static bool configured[64] = {};  // the attribute is per device
  const int dev = q.get_device();
  if (!configured[dev & 63]) {
    check_smem_optin(smem, dev, "fa_fwd_kernel");
    MINT_CUDA_CHECK(cudaFuncSetAttribute(fa::fa_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured[dev & 63] = true;
  }
  dim3 grid((T + fa::kTiles * fa::kBM - 1) / (fa::kTiles * fa::kBM), Hq, B);
  // O leaves in 32-row x 64-dim boxes, two TMA stores per softmax warp
  const CUtensorMap to = make_tmap_3d_bf16(o.data_ptr(), fa::kD, Hq, static_cast<uint64_t>(B) * T, fa::kD,
                                           static_cast<uint64_t>(Hq) * fa::kD, 64, 1, 32, true);
  fa::fa_fwd_kernel<<<grid, fa::kThreads, smem, at::cuda::getCurrentCUDAStream()>>>(tq, tk, tv, to, p);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return {o, lse};
}

}  // namespace mint
