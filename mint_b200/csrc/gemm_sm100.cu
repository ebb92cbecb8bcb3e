// Persistent, warp-specialized tcgen05 GEMM for sm_100a:  C = alpha * op(A) @ op(B) + beta * D.
//
// Layout: row-major with A [M,K] (K-major) or [K,M] (MN-major), B [N,K] (K-major) or [K,N]
// (MN-major); no operand is ever transposed in memory: the TMA boxes and the UMMA shared-memory
// descriptors describe either major-ness directly.
//
// One CTA per SM, 192 threads:
//   warp 0      TMA producer: 128B-swizzled A/B tiles (BK = 64) into a kStages-deep ring
//   warp 1      TMEM allocation + single-thread tcgen05.mma issue (M = 128, N = BN, K = 16)
//   warps 2..5  epilogue: tcgen05.ld of the fp32 accumulator (32 lanes x 32 columns per load),
//               alpha / beta*D, conversion and global stores
// The fp32 accumulator is double-buffered in tensor memory (2 x BN columns) so the epilogue of
// tile t overlaps the MMAs of tile t+1. Every mbarrier wait is bounded (common.cuh); on a
// timeout the kernel records a status code, drains its in-flight MMAs, frees TMEM and exits.
#include <cstdio>
#include <cstdlib>

#include "common.cuh"
#include "host_common.h"

namespace mint {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;

template <int BN>
struct Cfg {
  static constexpr int kStages = (BN == 256) ? 4 : 6;
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kBarrierBytes = 1024;
  static constexpr int kStagingBytes = 4 * 2 * 4096;  // 4 epilogue warps x 2 buffers x (32 x 32 fp32)
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + kBarrierBytes + kStagingBytes;
  static_assert(kSmemBytes <= 232448, "shared-memory layout exceeds the per-block opt-in limit");
};

struct Params {
  void* C;
  const void* D;
  int M, N, K;
  long long ldc, ldd;
  float alpha, beta;
  const float* alpha_ptr;
  int c_fp32, d_fp32;
  int tiles_m, tiles_n;
  int splits;      // split-K factor: work item = (tile, split)
  int kbps;        // k-blocks per split
  int atomic_out;  // C (fp32) += alpha * acc with 16-byte vector reductions
  int batch;       // independent GEMMs sharing shapes (operands / C addressed as 3-D TMA maps)
  long long sd;    // batch stride of D in elements
  int diag;        // timing diagnostics (MINT_GEMM_DIAG bits): 1 skip the epilogue body, 2 skip the MMAs,
                   // 4 skip the TMA loads (results are then meaningless; for isolating pipeline stages)
  uint32_t* status;
};

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& tm, int& tn) {
  constexpr int G = 8;  // groups of 8 M-tiles sweep all N-tiles: B tiles stay hot in L2
  const int per_group = G * tiles_n;
  const int group = tile / per_group;
  const int first_m = group * G;
  const int gsize = min(tiles_m - first_m, G);
  const int r = tile % per_group;
  tm = first_m + r % gsize;
  tn = r / gsize;
}

// work item -> (batch, tile m, tile n, first k-block, k-block count)
__device__ __forceinline__ void work_item(const Params& p, int w, int kblocks, int& bi, int& tm, int& tn, int& kb0,
                                          int& nkb) {
  const int tiles = p.tiles_m * p.tiles_n;
  const int per_batch = tiles * p.splits;
  bi = w / per_batch;
  w -= bi * per_batch;
  const int tile = w % tiles;
  const int split = w / tiles;
  tile_coords(tile, p.tiles_m, p.tiles_n, tm, tn);
  kb0 = split * p.kbps;
  nkb = min(kblocks, kb0 + p.kbps) - kb0;
}

// v[j] += beta * D[j] for the first n (<= 64) columns of one output row at element offset `off`
// (fp32 or bf16 D). Fully unrolled with constant indices so v stays in registers.
__device__ __forceinline__ void add_beta_d(const Params& p, long long off, float (&v)[64], int n) {
  if (p.d_fp32) {
    const float* dp = static_cast<const float*>(p.D) + off;
    if (n == 64) {
#pragma unroll
      for (int j = 0; j < 64; j += 4) {
        const float4 d4 = *reinterpret_cast<const float4*>(dp + j);
        v[j] += p.beta * d4.x;
        v[j + 1] += p.beta * d4.y;
        v[j + 2] += p.beta * d4.z;
        v[j + 3] += p.beta * d4.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        if (j < n) v[j] += p.beta * dp[j];
      }
    }
  } else {
    const __nv_bfloat16* dp = static_cast<const __nv_bfloat16*>(p.D) + off;
    if (n == 64) {
#pragma unroll
      for (int j = 0; j < 64; j += 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(dp + j);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          v[j + 2 * e] += p.beta * f.x;
          v[j + 2 * e + 1] += p.beta * f.y;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        if (j < n) v[j] += p.beta * __bfloat162float(dp[j]);
      }
    }
  }
}

// Epilogue of one accumulator tile for one warp: its 32 TMEM lanes (rows row0 .. row0+31 of C) x BN
// columns in 64-column groups: two tcgen05.ld per wait, alpha / beta*D, conversion into a 128B-
// swizzled shared-memory staging tile (double-buffered per warp, 4 KB) and TMA stores (one 32 x 64
// bf16 box, or two 32 x 32 fp32 boxes / TMA reduce-adds) that clip rows and columns outside C.
template <int BN>
__device__ __forceinline__ void epilogue_tile(const Params& p, const CUtensorMap* tmc, uint32_t tmem_acc, int row0,
                                              int col_base, int bi, float alpha, bool f32_out, uint8_t* bufs, int lane,
                                              int& seq) {
  const int row = row0 + lane;
  if (p.diag & 1) return;
#pragma unroll 1
  for (int g = 0; g < BN / 64; ++g) {
    uint32_t r0[32], r1[32];
    tmem_ld_32x32b_x32(tmem_acc + g * 64, r0);
    tmem_ld_32x32b_x32(tmem_acc + g * 64 + 32, r1);
    tmem_ld_wait();
    const int col0 = col_base + g * 64;
    if (col0 >= p.N || row0 >= p.M) continue;  // warp-uniform
    float v[64];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      v[j] = alpha * __uint_as_float(r0[j]);
      v[32 + j] = alpha * __uint_as_float(r1[j]);
    }
    if (p.D != nullptr && p.beta != 0.0f && row < p.M) {
      add_beta_d(p, bi * p.sd + static_cast<long long>(row) * p.ldd + col0, v, min(64, p.N - col0));
    }
    if (f32_out) {
      // two 32 x 32 fp32 boxes (128 B rows, 128B swizzle: chunk j of row `lane` at j ^ (lane % 8))
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        if (col0 + hh * 32 >= p.N) break;
        uint8_t* buf = bufs + (seq & 1) * 4096;
        if (lane == 0) bulk_wait_read<1>();  // the store issued two boxes ago read this buffer
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          *reinterpret_cast<float4*>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) =
              make_float4(v[hh * 32 + 4 * j], v[hh * 32 + 4 * j + 1], v[hh * 32 + 4 * j + 2], v[hh * 32 + 4 * j + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (p.atomic_out) {
            tma_reduce_add_3d(tmc, buf, col0 + hh * 32, row0, bi);
          } else {
            tma_store_3d(tmc, buf, col0 + hh * 32, row0, bi);
          }
          bulk_commit();
        }
        ++seq;
      }
    } else {
      // one 32 x 64 bf16 box (128 B rows, 128B swizzle)
      uint8_t* buf = bufs + (seq & 1) * 4096;
      if (lane == 0) bulk_wait_read<1>();
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint4 u;
        u.x = pack_bf16x2(v[8 * j], v[8 * j + 1]);
        u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
        u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
        u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
        *reinterpret_cast<uint4*>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) = u;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(tmc, buf, col0, row0, bi);
        bulk_commit();
      }
      ++seq;
    }
  }
}

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                const __grid_constant__ CUtensorMap tmc, Params p) {
  using C_ = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C_::kStages * C_::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C_::kStages * C_::kStageBytes);
  uint64_t* empty = full + C_::kStages;
  uint64_t* tfull = empty + C_::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* staging = smem + C_::kStages * C_::kStageBytes + C_::kBarrierBytes;  // 1024-aligned

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C_::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, C_::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.tiles_m * p.tiles_n * p.splits * p.batch;
  const int kblocks = (p.K + BK - 1) / BK;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tma);
      tma_prefetch_desc(&tmb);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int bi, tm, tn, kb0, nkb;
        work_item(p, tile, kblocks, bi, tm, tn, kb0, nkb);
        const int m0 = tm * BM, n0 = tn * BN;
        for (int kb = kb0; kb < kb0 + nkb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kStatusTimeoutProducer, abort_flag)) {
            ok = false;
            break;
          }
          if (p.diag & 4) {
            mbar_arrive(&full[stage]);
            if (++stage == C_::kStages) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          mbar_arrive_expect_tx(&full[stage], C_::kStageBytes);
          uint8_t* a_dst = sA + stage * C_::kABytes;
          uint8_t* b_dst = sB + stage * C_::kBBytes;
          const int k0 = kb * BK;
          if constexpr (!A_MN) {
            tma_load_3d(a_dst, &tma, &full[stage], k0, m0, bi);
          } else {
#pragma unroll
            for (int i = 0; i < BM / 64; ++i) tma_load_3d(a_dst + i * 8192, &tma, &full[stage], m0 + i * 64, k0, bi);
          }
          if constexpr (!B_MN) {
            tma_load_3d(b_dst, &tmb, &full[stage], k0, n0, bi);
          } else {
#pragma unroll
            for (int i = 0; i < BN / 64; ++i) tma_load_3d(b_dst + i * 8192, &tmb, &full[stage], n0 + i * 64, k0, bi);
          }
          if (++stage == C_::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // let any TMA copy already in flight land before the CTA's shared memory goes away
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++t) {
        const int acc = t & 1;
        const uint32_t acc_phase = (t >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.status, kStatusTimeoutMma, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        int bi_, tm_, tn_, kb0, nkb;
        work_item(p, tile, kblocks, bi_, tm_, tn_, kb0, nkb);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status, kStatusTimeoutMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * C_::kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * C_::kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // K-major SW128: step 16 elements = 32 bytes inside the swizzle atom (SBO = 8 rows x 128 B).
            // MN-major SW128: step 16 K-rows = 2048 bytes; LBO = 8 KB between 64-wide MN atoms.
            const uint64_t adesc = A_MN ? umma_desc_sw128(a_addr + k * 2048, 8192, 1024)
                                        : umma_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? umma_desc_sw128(b_addr + k * 2048, 8192, 1024)
                                        : umma_desc_sw128(b_addr + k * 32, 16, 1024);
            if (!(p.diag & 2)) umma_bf16(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == C_::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
      // drain: every MMA issued by this thread completes before TMEM is released
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, p.status, kStatusTimeoutMma, nullptr);
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane quadrant (warp % 4). Each 32x32 accumulator chunk is converted
    // in registers, written to a swizzled shared-memory staging buffer (double-buffered per warp)
    // and written out by one TMA store (or TMA reduce-add for accumulating GEMMs); TMA clips rows
    // and columns outside C.
    const int q = warp & 3;
    uint8_t* bufs = staging + (warp - 2) * 2 * 4096;
    float alpha = p.alpha;
    if (p.alpha_ptr != nullptr) alpha *= *p.alpha_ptr;
    const bool f32_out = p.c_fp32 || p.atomic_out;
    int t = 0;
    int seq = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t) {
      const int acc = t & 1;
      const uint32_t acc_phase = (t >> 1) & 1;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, p.status, kStatusTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      int bi, tm, tn, kb0_, nkb_;
      work_item(p, tile, kblocks, bi, tm, tn, kb0_, nkb_);
      const int row0 = tm * BM + q * 32;
      epilogue_tile<BN>(p, &tmc, tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN, row0, tn * BN, bi,
                        alpha, f32_out, bufs, lane, seq);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C_::kTmemCols);
  }
}

template <int BN, bool A_MN, bool B_MN>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const Params& p, int sms,
            cudaStream_t stream) {
  using C_ = Cfg<BN>;
  auto kern = gemm_kernel<BN, A_MN, B_MN>;
  static bool configured[64] = {};  // the attribute is per device
  int dev = 0;
  MINT_CUDA_CHECK(cudaGetDevice(&dev));
  if (!configured[dev & 63]) {
    check_smem_optin(C_::kSmemBytes, dev, "gemm");
    MINT_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::kSmemBytes));
    configured[dev & 63] = true;
  }
  const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n * p.splits * p.batch;
  const int grid = tiles < sms ? static_cast<int>(tiles) : sms;
  kern<<<grid, kThreads, C_::kSmemBytes, stream>>>(ta, tb, tc, p);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

// ---------------------------------------------------------------------------------------------
// Tensor-parallel communication fused into the CTA-pair GEMM (rows of A / C are tokens).
// A rank's token chunk is made of segments of `seg` rows: segment s of rank p holds gathered rows
// [(s * world + p) * seg, ... + seg) (sequence parallelism shards every sequence of a batch).
//   COMM 1, all-gather -> GEMM: A is this rank's symmetric gathered buffer; its own chunk is already
//     in place. Copy warps pull the peers' chunks (128-row blocks, claimed dynamically) over NVLink
//     into it and publish a per-block flag; the TMA producer waits for a block's flag before
//     loading it. This rank's own rows are scheduled first, so compute starts at once.
//   COMM 2, GEMM -> reduce-scatter: tiles of peers' chunks are computed first; the epilogue stages
//     each 32 x 64 piece in shared memory and a TMA store (one tensor map per peer over that peer's
//     receive slot for this rank) carries it over NVLink, so the epilogue warps never wait on remote
//     stores. A warp publishes a tile's flag once the tile's stores are complete, two tiles behind
//     the newest. This rank's own tiles come last; their epilogue adds the received partials before
//     the TMA store of the reduced rows (C then covers only this rank's chunk, in local row order).
// Every call has a sequence number `seq`; flags hold the seq of the call that set them and are
// never reset. At its start each rank writes seq into every peer's arrive[rank]; no rank reads or
// writes a peer's buffers of call seq before seeing that peer arrive at seq.
struct CommParams {
  CUtensorMap rs_push_map[8];    // RS: peer p's receive slot for this rank as a TMA store map ([Mc, N] bf16)
  int rank, world, seg, seq;
  int* arrive_local;             // [world] (symmetric): arrive_local[p] = latest call rank p entered
  int* arrive_peer[8];           // peers' arrive arrays
  const uint8_t* ag_src[8];      // AG: peers' gathered buffers (same layout and offset as ours)
  uint8_t* ag_dst;               // AG: our gathered buffer (the A operand)
  long long ag_row_bytes;        // AG: bytes per row of A
  int* rowflag;                  // AG: [M / 128] local flags (seq when a block landed)
  int* blockcnt;                 // AG: [M / 128] local piece counters (+kAgPieces per block per call, never reset)
  unsigned long long* claim;     // AG: work counter, zero at launch
  __nv_bfloat16* rs_push[8];     // RS: peer p's receive slot for this rank ([Mc, N], rows of chunk p)
  const __nv_bfloat16* rs_recv;  // RS: our receive slots [world][Mc, N]
  int* rs_flag_peer[8];          // RS: peer p's flags for this rank [Mc / 128][tiles_n][4]
  const int* rs_flag_local;      // RS: our flags [world][rs_flag_stride], block of source s at s * stride
  long long rs_flag_stride;      // RS: flags per source rank (>= Mc / 128 * tiles_n * 4)
  long long mc;                  // rows per chunk (M / world)
  int rs_lag;                    // RS: own tile k follows the peers' tile k by this many 256-row tiles
  // GeGLU modes (COMM 3 forward, 4 backward; no communication)
  CUtensorMap geglu_map;         // 3: h [M, F] store map (32 x 64 bf16 boxes)
  const __nv_bfloat16* geglu_ab; // 4: the forward's [a | b] rows [M, 2F] (read by the epilogue)
  int geglu_f;                   // F (hidden width; multiple of 128)
};

__device__ __forceinline__ int chunk_of_row(const CommParams& c, long long g) {
  return static_cast<int>((g / c.seg) % c.world);
}
__device__ __forceinline__ long long local_row_of(const CommParams& c, long long g) {
  return (g / (static_cast<long long>(c.seg) * c.world)) * c.seg + g % c.seg;
}
__device__ __forceinline__ long long gathered_row_of(const CommParams& c, int p, long long l) {
  return ((l / c.seg) * c.world + p) * c.seg + l % c.seg;
}
// 256-row tile ordinal -> tile index.
// All-gather: own chunk first (its rows are local), then the peers' chunks in rotation order.
// Reduce-scatter: peers' tiles and own tiles interleaved, so the pushes over NVLink spread over the
// whole kernel instead of filling its first half: local tile index li contributes the peers' tiles
// li and then this rank's own tile li - D (D = min(rs_lag, tiles per chunk); rs_lag = 8 by default:
// one tile group of the schedule), the remaining own tiles come last. Every rank uses the same order, so a peer pushes
// the partial of own tile k at an earlier ordinal than the one at which this rank reduces tile k.
__device__ __forceinline__ int comm_tile_m(const CommParams& c, int o, int tiles_m2, bool own_first) {
  const int w = c.world;
  const int tpc = tiles_m2 / w;  // 256-row tiles per chunk
  int p, li;
  if (own_first) {
    const int cp = o / tpc;
    p = (c.rank + cp) % w;
    li = o % tpc;
  } else {
    const int D = min(c.rs_lag, tpc);
    const int head = D * (w - 1);
    if (o < head) {
      li = o / (w - 1);
      p = (c.rank + 1 + o % (w - 1)) % w;
    } else if (o - head < (tpc - D) * w) {
      const int o2 = o - head;
      const int k = o2 % w;
      if (k < w - 1) {
        li = D + o2 / w;
        p = (c.rank + 1 + k) % w;
      } else {
        li = o2 / w;  // own tile (D + o2 / w) - D
        p = c.rank;
      }
    } else {
      li = tpc - D + (o - head - (tpc - D) * w);
      p = c.rank;
    }
  }
  const long long l = static_cast<long long>(li) * 256;  // local row of the tile's first row
  return static_cast<int>(gathered_row_of(c, p, l) / 256);
}

// RS epilogue of one warp's 32 rows x BN columns: push to the owner, or reduce and store.
constexpr int kRsPend = 16;  // room of the per-warp queue of pushed tiles whose flags are pending
constexpr int kRsLag = 2;    // a pushed tile's flag is released once two newer tiles were pushed

// Publish the flags of every tile this warp pushed: wait until all of this lane's TMA stores have
// been performed, order them (async proxy, then system scope) before the releases.
// (No separate system fence: `st.release.sys` already orders every earlier write of the thread;
// one per tile measured 1.3 ms of 4.6 at M=131072 N=8192 tp=2.)
__device__ __forceinline__ void rs_flush_lane0(const CommParams& c, const int* pend, int& npend) {
  if (npend == 0) return;
  bulk_wait_all();
  fence_proxy_async_global();
  for (int i = 0; i < npend; ++i) st_release_sys(c.rs_flag_peer[pend[2 * i]] + pend[2 * i + 1], c.seq);
  npend = 0;
}
__device__ __forceinline__ void rs_flush(const CommParams& c, int* pend, int& npend, int lane) {
  if (lane == 0) rs_flush_lane0(c, pend, npend);
  __syncwarp();
  npend = 0;
}

// After a push of kG bulk groups: release the oldest pending tile once only the kRsLag newest tiles
// (kRsLag * kG groups, every tile commits exactly kG) may still be in flight.
template <int kG>
__device__ __forceinline__ void rs_release_lagged(const CommParams& c, int* pend, int& npend, int lane) {
  if (npend <= kRsLag) return;
  if (lane == 0) {
    bulk_wait<kRsLag * kG>();
    fence_proxy_async_global();
    st_release_sys(c.rs_flag_peer[pend[0]] + pend[1], c.seq);
    for (int i = 1; i < npend; ++i) {
      pend[2 * (i - 1)] = pend[2 * i];
      pend[2 * (i - 1) + 1] = pend[2 * i + 1];
    }
  }
  __syncwarp();
  --npend;
}

template <int BN>
__device__ __forceinline__ bool epilogue_tile_rs(const Params& p, const CommParams& c, const CUtensorMap* tmc,
                                                 uint32_t tmem_acc, long long grow0, int tn, int q, float alpha,
                                                 uint8_t* bufs, int lane, int& seq, volatile int* abort_flag,
                                                 int* pend, int& npend) {
  const int chunk = chunk_of_row(c, grow0);
  const long long lrow0 = local_row_of(c, grow0);
  const int tiles_n = (p.N + BN - 1) / BN;
  const long long fidx = ((lrow0 / 128) * tiles_n + tn) * 4 + q;
  const int col_base = tn * BN;
  if (chunk != c.rank) {
    // the owner entered this call: its receive slot is free
    bool ok = true;
    if (lane == 0) ok = wait_flag(&c.arrive_local[chunk], c.seq, true, p.status, kStatusTimeoutPeer, abort_flag);
    if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
    const CUtensorMap* pmap = &c.rs_push_map[chunk];
#pragma unroll 1
    for (int g = 0; g < BN / 64; ++g) {
      uint32_t r0[32], r1[32];
      tmem_ld_32x32b_x32(tmem_acc + g * 64, r0);
      tmem_ld_32x32b_x32(tmem_acc + g * 64 + 32, r1);
      tmem_ld_wait();
      const int col0 = col_base + g * 64;
      if (col0 < p.N) {
        uint8_t* buf = bufs + (seq & 1) * 4096;
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 u;
          u.x = pack_bf16x2(alpha * __uint_as_float(r0[8 * j]), alpha * __uint_as_float(r0[8 * j + 1]));
          u.y = pack_bf16x2(alpha * __uint_as_float(r0[8 * j + 2]), alpha * __uint_as_float(r0[8 * j + 3]));
          u.z = pack_bf16x2(alpha * __uint_as_float(r0[8 * j + 4]), alpha * __uint_as_float(r0[8 * j + 5]));
          u.w = pack_bf16x2(alpha * __uint_as_float(r0[8 * j + 6]), alpha * __uint_as_float(r0[8 * j + 7]));
          *reinterpret_cast<uint4*>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) = u;
          u.x = pack_bf16x2(alpha * __uint_as_float(r1[8 * j]), alpha * __uint_as_float(r1[8 * j + 1]));
          u.y = pack_bf16x2(alpha * __uint_as_float(r1[8 * j + 2]), alpha * __uint_as_float(r1[8 * j + 3]));
          u.z = pack_bf16x2(alpha * __uint_as_float(r1[8 * j + 4]), alpha * __uint_as_float(r1[8 * j + 5]));
          u.w = pack_bf16x2(alpha * __uint_as_float(r1[8 * j + 6]), alpha * __uint_as_float(r1[8 * j + 7]));
          *reinterpret_cast<uint4*>(buf + lane * 128 + (((j + 4) ^ (lane & 7)) << 4)) = u;
        }
        fence_proxy_async_smem();
        __syncwarp();
        // the owner's receive slot for this rank: rows lrow0.. of chunk-local order, columns col0..
        if (lane == 0) tma_store_3d(pmap, buf, col0, static_cast<int>(lrow0), 0);
        ++seq;
      }
      if (lane == 0) bulk_commit();  // exactly BN / 64 groups per tile (empty past N) for the lag count
    }
    if (lane == 0) {
      pend[2 * npend] = chunk;
      pend[2 * npend + 1] = static_cast<int>(fidx);
    }
    __syncwarp();
    ++npend;
    rs_release_lagged<BN / 64>(c, pend, npend, lane);
    return true;
  }
  // own rows: wait for every peer's partial of these 32 rows, reduce and store. A warp that has to
  // wait first publishes every tile it pushed (a peer may be waiting on one of them), so no two
  // ranks can wait on each other; when the partials are already there, its pushes stay in flight.
  bool ok = true;
  if (lane == 0) {
    bool ready = true;
    for (int src = 0; src < c.world && ready; ++src) {
      if (src != c.rank) ready = ld_acquire_sys(c.rs_flag_local + src * c.rs_flag_stride + fidx) >= c.seq;
    }
    if (!ready) {
      rs_flush_lane0(c, pend, npend);
      for (int src = 0; src < c.world && ok; ++src) {
        if (src == c.rank) continue;
        ok = wait_flag(c.rs_flag_local + src * c.rs_flag_stride + fidx, c.seq, true, p.status, kStatusTimeoutPeer,
                       abort_flag);
      }
    }
  }
  npend = __shfl_sync(0xffffffffu, npend, 0);
  if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
  const long long lrow = lrow0 + lane;
#pragma unroll 1
  for (int g = 0; g < BN / 64; ++g) {
    uint32_t r0[32], r1[32];
    tmem_ld_32x32b_x32(tmem_acc + g * 64, r0);
    tmem_ld_32x32b_x32(tmem_acc + g * 64 + 32, r1);
    tmem_ld_wait();
    const int col0 = col_base + g * 64;
    if (col0 >= p.N) continue;
    float v[64];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      v[j] = alpha * __uint_as_float(r0[j]);
      v[32 + j] = alpha * __uint_as_float(r1[j]);
    }
    if (lrow < c.mc && col0 + 64 <= p.N) {
      for (int src = 0; src < c.world; ++src) {
        if (src == c.rank) continue;
        const __nv_bfloat16* rp = c.rs_recv + src * c.mc * p.N + lrow * p.N + col0;
#pragma unroll
        for (int j = 0; j < 64; j += 8) {
          const uint4 u = *reinterpret_cast<const uint4*>(rp + j);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(h[e]);
            v[j + 2 * e] += f.x;
            v[j + 2 * e + 1] += f.y;
          }
        }
      }
    } else if (lrow < c.mc) {
      for (int src = 0; src < c.world; ++src) {
        if (src == c.rank) continue;
        const __nv_bfloat16* rp = c.rs_recv + src * c.mc * p.N + lrow * p.N + col0;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          if (col0 + j < p.N) v[j] += __bfloat162float(rp[j]);
        }
      }
    }
    uint8_t* buf = bufs + (seq & 1) * 4096;
    if (lane == 0) bulk_wait_read<1>();
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint4 u;
      u.x = pack_bf16x2(v[8 * j], v[8 * j + 1]);
      u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
      u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
      u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
      *reinterpret_cast<uint4*>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) = u;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(tmc, buf, col0, static_cast<int>(lrow0), 0);
      bulk_commit();
    }
    ++seq;
  }
  return true;
}

// ---------------------------------------------------------------------------------------------
// GeGLU fused into the fc1||fc2 GEMM and into the fc3 input-gradient GEMM.
// gelu_tanh(x) = 0.5 x (1 + tanh(k0 (x + k1 x^3))), k0 = sqrt(2 / pi), k1 = 0.044715
constexpr float kGeluK0 = 0.7978845608028654f;
constexpr float kGeluK1 = 0.044715f;

// Stage 32 rows x 64 bf16 columns (this lane's row in v[0..63]) in a 128B-swizzled 4 KB buffer of
// the per-warp double buffer and store it with one TMA box at (x, y).
__device__ __forceinline__ void stage_store_bf16(const CUtensorMap* map, const float* v, uint8_t* bufs, int lane,
                                                 int& seq, int x, int y) {
  uint8_t* buf = bufs + (seq & 1) * 4096;
  if (lane == 0) bulk_wait_read<1>();  // the store issued two boxes ago has read this buffer
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint4 u;
    u.x = pack_bf16x2(v[8 * j], v[8 * j + 1]);
    u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
    u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
    u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
    *reinterpret_cast<uint4*>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) = u;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_3d(map, buf, x, y, 0);
    bulk_commit();
  }
  ++seq;
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// tanh as the single-instruction hardware approximation (relative error ~2^-11, far below the bf16
// rounding of the values it feeds)
__device__ __forceinline__ float tanh_hw(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Forward (COMM 3): the pair's B rows are fc1 rows [tn * BN/2, +BN/2) (leader) and fc2 rows
// [F + tn * BN/2, +BN/2) (follower), so accumulator columns [0, BN/2) hold a and [BN/2, BN) hold
// the matching b. The epilogue stores a and b into their places of ab [M, 2F] (kept for the
// backward) and h = gelu_tanh(a) * b into h [M, F], from the bf16-rounded a and b (the same
// values a separate GeGLU pass over the stored ab would read).
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile_geglu_fwd(const Params& p, const CommParams& c, const CUtensorMap* tmc,
                                                        uint32_t tmem_acc, int row0, int tn, int half, uint8_t* bufs,
                                                        int lane, int& seq) {
  // EPI 4: one warp per lane quadrant takes every 64-column group of a; EPI 8: two warps, one group each
  static_assert(BN == 256 && (EPI == 4 || EPI == 8), "GeGLU forward epilogue layout");
  const int F = c.geglu_f;
  constexpr int kGroups = EPI == 4 ? BN / 128 : 1;
#pragma unroll 1
  for (int gi = 0; gi < kGroups; ++gi) {
    const int g = EPI == 4 ? gi : half;
    uint32_t ra[2][32], rb[2][32];
    tmem_ld_32x32b_x32(tmem_acc + g * 64, ra[0]);
    tmem_ld_32x32b_x32(tmem_acc + g * 64 + 32, ra[1]);
    tmem_ld_32x32b_x32(tmem_acc + BN / 2 + g * 64, rb[0]);
    tmem_ld_32x32b_x32(tmem_acc + BN / 2 + g * 64 + 32, rb[1]);
    tmem_ld_wait();
    const int col0 = tn * (BN / 2) + g * 64;
    if (col0 >= F || row0 >= p.M || (p.diag & 1)) continue;  // warp-uniform
    float v[64];
#pragma unroll
    for (int j = 0; j < 64; ++j) v[j] = bf16_round(__uint_as_float(ra[j >> 5][j & 31]));
    stage_store_bf16(tmc, v, bufs, lane, seq, col0, row0);
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const float b = bf16_round(__uint_as_float(rb[j >> 5][j & 31]));
      const float a = v[j];
      v[j] = b;
      ra[j >> 5][j & 31] = __float_as_uint(0.5f * a * (1.f + tanh_hw(kGeluK0 * (a + kGeluK1 * a * a * a))) * b);
    }
    stage_store_bf16(tmc, v, bufs, lane, seq, F + col0, row0);
#pragma unroll
    for (int j = 0; j < 64; ++j) v[j] = __uint_as_float(ra[j >> 5][j & 31]);
    stage_store_bf16(&c.geglu_map, v, bufs, lane, seq, col0, row0);
  }
}

// Backward (COMM 4): the GEMM computes dh = dy @ W3 ([M, F]); for each 64-column group the
// epilogue reads the forward's a and b of its 32 rows, rounds dh to bf16 (the value a separate pass
// would read) and stores da = dh * b * gelu'(a) and db = dh * gelu(a) into dab [M, 2F]; dh itself
// never reaches memory.
template <int BN>
__device__ __forceinline__ void epilogue_tile_geglu_bwd(const Params& p, const CommParams& c, const CUtensorMap* tmc,
                                                        uint32_t tmem_acc, int row0, int col_base, uint8_t* bufs,
                                                        int lane, int& seq) {
  const int F = c.geglu_f;
  const int row = row0 + lane;
#pragma unroll 1
  for (int g = 0; g < BN / 128; ++g) {  // this warp's half of the tile's columns
    const int col0 = col_base + g * 64;
    uint4 ua[8], ub[8];
    const bool live = col0 < F && row0 < p.M && !(p.diag & 1);  // warp-uniform
    if (live && row < p.M) {
      const __nv_bfloat16* arow = c.geglu_ab + static_cast<long long>(row) * 2 * F + col0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        ua[j] = *reinterpret_cast<const uint4*>(arow + 8 * j);
        ub[j] = *reinterpret_cast<const uint4*>(arow + F + 8 * j);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) ua[j] = ub[j] = make_uint4(0u, 0u, 0u, 0u);
    }
    uint32_t r[2][32];
    tmem_ld_32x32b_x32(tmem_acc + g * 64, r[0]);
    tmem_ld_32x32b_x32(tmem_acc + g * 64 + 32, r[1]);
    tmem_ld_wait();
    if (!live) continue;
    // da and db go straight into the two staging buffers, 8 columns at a time (both buffers free
    // once every earlier store of this warp has read its source)
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
    uint8_t* bufa = bufs;
    uint8_t* bufb = bufs + 4096;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&ua[j]);
      const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&ub[j]);
      uint32_t qa[4], qb[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 a2 = __bfloat1622float2(pa[e]);
        const float2 b2 = __bfloat1622float2(pb[e]);
        const float av[2] = {a2.x, a2.y}, bv[2] = {b2.x, b2.y};
        float da[2], db[2];
#pragma unroll
        for (int z = 0; z < 2; ++z) {
          const int k = 8 * j + 2 * e + z;
          const float x = av[z];
          const float gr = bf16_round(__uint_as_float(r[k >> 5][k & 31]));
          const float t = tanh_hw(kGeluK0 * (x + kGeluK1 * x * x * x));
          const float gelu = 0.5f * x * (1.f + t);
          const float dgelu = 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * kGeluK0 * (1.f + 3.f * kGeluK1 * x * x);
          da[z] = gr * bv[z] * dgelu;
          db[z] = gr * gelu;
        }
        qa[e] = pack_bf16x2(da[0], da[1]);
        qb[e] = pack_bf16x2(db[0], db[1]);
      }
      const int off = lane * 128 + ((j ^ (lane & 7)) << 4);
      *reinterpret_cast<uint4*>(bufa + off) = make_uint4(qa[0], qa[1], qa[2], qa[3]);
      *reinterpret_cast<uint4*>(bufb + off) = make_uint4(qb[0], qb[1], qb[2], qb[3]);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(tmc, bufa, col0, row0, 0);
      tma_store_3d(tmc, bufb, F + col0, row0, 0);
      bulk_commit();
    }
    seq += 2;
  }
}

constexpr int kAgPieces = 8;  // a 128-row block is copied as 8 pieces of 16 rows by different warps

// ---------------------------------------------------------------------------------------------
// CTA-pair kernel: a cluster of 2 CTAs on 2 SMs computes one 256 x BN tile with tcgen05.mma
// cta_group::2. CTA r of the pair loads rows [128 r, 128 r + 128) of the A tile and rows
// [BN/2 r, BN/2 r + BN/2) of the B tile into its own shared memory; the leader (r = 0) issues
// the MMAs, which read both CTAs' halves and write 128 rows of the accumulator into each CTA's
// tensor memory. Each SM thus streams 16 KB of A and BN/8 KB of B per 64-deep k-block instead
// of 16 + BN/4 KB, halving the shared operand traffic the single-CTA kernel spends on B.
// Barriers: full[s] and tempty[] live in the leader (the follower's TMA completes bytes on the
// leader's full[s]; both epilogues arrive on the leader's tempty[]); empty[s] and tfull[] live in
// both CTAs and the leader's MMA thread commits to each explicitly.
template <int BN, int EPI = 4>
struct Cfg2 {
  static constexpr int kStages = EPI == 8 ? 5 : 6;   // 192 KB of operands in flight per SM (160 with 8 epilogue warps)
  static constexpr int kABytes = 128 * BK * 2;       // this CTA's 128 rows of A
  static constexpr int kBBytes = (BN / 2) * BK * 2;  // this CTA's BN/2 rows of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kBarrierBytes = 1024;  // barriers, TMEM slot, abort flag; bytes 256..767 RS flag queues
  // epilogue warps: 4 (one per TMEM lane quadrant) or 8 (two per quadrant, half the columns each);
  // measured alike for plain epilogues, so those keep a sixth operand stage; the GeGLU backward
  // epilogue (two global loads and a transcendental per element) uses 8
  static constexpr int kEpiWarps = EPI;
  static constexpr int kThreads = (2 + kEpiWarps) * 32;
  static constexpr int kCopyWarps = 2;  // all-gather mode: warps pulling peers' rows
  static constexpr int kStagingBytes = kEpiWarps * 2 * 4096;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + kBarrierBytes + kStagingBytes;
  static_assert(kSmemBytes <= 232448, "shared-memory layout exceeds the per-block opt-in limit");
};

template <int COMM>
constexpr int pair_epi_warps() {
  return COMM == 4 ? 8 : 4;  // the GeGLU backward epilogue (loads + transcendentals) gets two warps per quadrant
}

template <int BN, int COMM>
constexpr int pair_threads() {
  using C_ = Cfg2<BN, pair_epi_warps<COMM>()>;
  return C_::kThreads + (COMM == 1 ? C_::kCopyWarps * 32 : 0);
}

template <int BN, bool A_MN, bool B_MN, int COMM>
__global__ void __launch_bounds__(pair_threads<BN, COMM>(), 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                     const __grid_constant__ CUtensorMap tmc, Params p, const __grid_constant__ CommParams c) {
  using C_ = Cfg2<BN, pair_epi_warps<COMM>()>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C_::kStages * C_::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C_::kStages * C_::kStageBytes);
  uint64_t* empty = full + C_::kStages;
  uint64_t* tfull = empty + C_::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* staging = smem + C_::kStages * C_::kStageBytes + C_::kBarrierBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cr = cluster_ctarank();
  const bool leader = cr == 0;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int st = 0; st < C_::kStages; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 2 * C_::kEpiWarps);  // every epilogue warp of both CTAs of the pair
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, C_::kTmemCols);
  constexpr bool kTP = COMM == 1 || COMM == 2;  // modes that talk to peers
  if (kTP && blockIdx.x == 0 && threadIdx.x == 64) {
    // this rank entered call seq: its inputs of the call are in place (stream order) and the buffers
    // peers write into for this call are no longer read by an earlier call
    __threadfence_system();
    for (int q = 0; q < c.world; ++q) {
      if (q != c.rank) st_release_sys(c.arrive_peer[q] + c.rank, c.seq);
    }
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialized before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles_m2 = (p.M + 255) / 256;
  const int tiles_per_batch = tiles_m2 * p.tiles_n * p.splits;
  const int num_tiles = tiles_per_batch * p.batch;
  const int kblocks = (p.K + BK - 1) / BK;
  // work item -> (batch, 256-row tile, column tile, k range)
  auto item = [&](int w, int& bi, int& tm, int& tn, int& kb0, int& nkb) {
    bi = w / tiles_per_batch;
    w -= bi * tiles_per_batch;
    const int tiles = tiles_m2 * p.tiles_n;
    const int tile = w % tiles;
    const int split = w / tiles;
    tile_coords(tile, tiles_m2, p.tiles_n, tm, tn);
    if constexpr (kTP) tm = comm_tile_m(c, tm, tiles_m2, COMM == 1);
    kb0 = split * p.kbps;
    nkb = min(kblocks, kb0 + p.kbps) - kb0;
  };

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tma);
      tma_prefetch_desc(&tmb);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int w = pair; w < num_tiles && ok; w += npairs) {
        int bi, tm, tn, kb0, nkb;
        item(w, bi, tm, tn, kb0, nkb);
        const int m0 = tm * 256 + static_cast<int>(cr) * 128;
        // GeGLU forward: the leader loads fc1 rows, the follower the matching fc2 rows (F below them)
        const int n0 = COMM == 3 ? static_cast<int>(cr) * c.geglu_f + tn * (BN / 2)
                                 : tn * BN + static_cast<int>(cr) * (BN / 2);
        if constexpr (COMM == 1) {
          // a peer's rows: wait until a copy warp has landed this 128-row block in our buffer
          if (chunk_of_row(c, m0) != c.rank) {
            if (!wait_flag(c.rowflag + m0 / 128, c.seq, false, p.status, kStatusTimeoutPeer, abort_flag)) {
              ok = false;
              break;
            }
            fence_proxy_async_global();
          }
        }
        for (int kb = kb0; kb < kb0 + nkb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kStatusTimeoutProducer, abort_flag)) {
            ok = false;
            break;
          }
          // the leader's full[stage] counts both CTAs' bytes; only the leader arrives on it
          if (p.diag & 4) {
            if (leader) mbar_arrive(&full[stage]);
            if (++stage == C_::kStages) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C_::kStageBytes);
          const uint32_t bar = mapa_shared(&full[stage], 0);
          uint8_t* a_dst = sA + stage * C_::kABytes;
          uint8_t* b_dst = sB + stage * C_::kBBytes;
          const int k0 = kb * BK;
          if constexpr (!A_MN) {
            tma_load_3d_pair(a_dst, &tma, bar, k0, m0, bi);
          } else {
#pragma unroll
            for (int i = 0; i < 2; ++i) tma_load_3d_pair(a_dst + i * 8192, &tma, bar, m0 + i * 64, k0, bi);
          }
          if constexpr (!B_MN) {
            tma_load_3d_pair(b_dst, &tmb, bar, k0, n0, bi);
          } else {
#pragma unroll
            for (int i = 0; i < BN / 128; ++i) tma_load_3d_pair(b_dst + i * 8192, &tmb, bar, n0 + i * 64, k0, bi);
          }
          if (++stage == C_::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = umma_idesc_bf16(256, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      bool ok = true;
      for (int w = pair; w < num_tiles && ok; w += npairs, ++t) {
        const int acc = t & 1;
        const uint32_t acc_phase = (t >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.status, kStatusTimeoutMma, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        int bi_, tm_, tn_, kb0, nkb;
        item(w, bi_, tm_, tn_, kb0, nkb);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status, kStatusTimeoutMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * C_::kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * C_::kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = A_MN ? umma_desc_sw128(a_addr + k * 2048, 8192, 1024)
                                        : umma_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? umma_desc_sw128(b_addr + k * 2048, 8192, 1024)
                                        : umma_desc_sw128(b_addr + k * 32, 16, 1024);
            if (!(p.diag & 2)) umma_bf16_pair(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(mapa_shared(&empty[stage], 0));
          umma_commit_pair(mapa_shared(&empty[stage], 1));
          if (++stage == C_::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) {
          umma_commit_pair(mapa_shared(&tfull[acc], 0));
          umma_commit_pair(mapa_shared(&tfull[acc], 1));
        }
      }
      umma_commit_pair(mapa_shared(mma_done, 0));
      mbar_wait(mma_done, 0, p.status, kStatusTimeoutMma, nullptr);
    }
  } else if (COMM == 1 && warp >= 2 + C_::kEpiWarps) {
    // copy warps: pull the peers' chunks into our gathered buffer in 16-row pieces (claimed
    // dynamically, peers in rotation order after this rank, blocks in the order the tile schedule
    // consumes them); the warp finishing the last piece of a 128-row block publishes its flag
    const long long blocks_per_chunk = c.mc / 128;
    const long long units = (c.world - 1) * blocks_per_chunk * kAgPieces;
    const long long n16 = 16 * c.ag_row_bytes / 16;  // 16-byte words per piece
    for (;;) {
      long long unit = 0;
      if (lane == 0) unit = static_cast<long long>(atomicAdd(c.claim, 1ull));
      unit = __shfl_sync(0xffffffffu, unit, 0);
      if (unit >= units || *abort_flag) break;
      const long long blk = unit / kAgPieces;
      const int piece = static_cast<int>(unit % kAgPieces);
      const int src = (c.rank + 1 + static_cast<int>(blk / blocks_per_chunk)) % c.world;
      const long long g0 = gathered_row_of(c, src, (blk % blocks_per_chunk) * 128);
      bool ok = true;
      if (lane == 0) ok = wait_flag(c.arrive_local + src, c.seq, true, p.status, kStatusTimeoutPeer, abort_flag);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      const long long r0 = g0 + piece * 16;
      const uint4* from = reinterpret_cast<const uint4*>(c.ag_src[src] + r0 * c.ag_row_bytes);
      uint4* to = reinterpret_cast<uint4*>(c.ag_dst + r0 * c.ag_row_bytes);
      for (long long i = lane; i < n16; i += 32 * 16) {
        uint4 v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          if (i + u * 32 < n16) v[u] = from[i + u * 32];
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          if (i + u * 32 < n16) to[i + u * 32] = v[u];
        }
      }
      fence_proxy_async_global();
      __syncwarp();
      if (lane == 0) {
        const int old = atom_add_acq_rel_gpu(c.blockcnt + g0 / 128, 1);
        if ((old + 1) % kAgPieces == 0) st_release_gpu(c.rowflag + g0 / 128, c.seq);
      }
    }
  } else {
    // warp w drains TMEM lane quadrant w % 4 (the lanes a warp may access), columns of half (w - 2) / 4
    const int q = warp & 3;
    const int half = C_::kEpiWarps == 8 ? (warp - 2) >> 2 : 0;
    constexpr int kCols = C_::kEpiWarps == 8 ? BN / 2 : BN;
    uint8_t* bufs = staging + (warp - 2) * 2 * 4096;
    float alpha = p.alpha;
    if (p.alpha_ptr != nullptr) alpha *= *p.alpha_ptr;
    const bool f32_out = p.c_fp32 || p.atomic_out;
    const uint32_t tempty_leader[2] = {mapa_shared(&tempty[0], 0), mapa_shared(&tempty[1], 0)};
    // reduce-scatter: flags of pushed tiles held back until a fence (in the barrier region's spare bytes)
    int* pend = reinterpret_cast<int*>(smem + C_::kStages * C_::kStageBytes + 256) + (warp - 2) * 2 * kRsPend;
    int npend = 0;
    int t = 0;
    int seq = 0;
    for (int w = pair; w < num_tiles; w += npairs, ++t) {
      const int acc = t & 1;
      const uint32_t acc_phase = (t >> 1) & 1;
      if constexpr (COMM == 2) {
        // the next accumulator may depend (through the MMA and the other epilogue warps) on a peer
        // that waits for a tile this warp pushed: publish them all before blocking on it
        if (__any_sync(0xffffffffu, npend > 0 && !mbar_try_wait(smem_u32(&tfull[acc]), acc_phase))) {
          rs_flush(c, pend, npend, lane);
        }
      }
      if (!mbar_wait_warp(&tfull[acc], acc_phase, p.status, kStatusTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      int bi, tm, tn, kb0_, nkb_;
      item(w, bi, tm, tn, kb0_, nkb_);
      const int row0 = tm * 256 + static_cast<int>(cr) * 128 + q * 32;
      if constexpr (COMM == 2) {
        const bool ok = epilogue_tile_rs<BN>(p, c, &tmc, tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN,
                                             row0, tn, q, alpha, bufs, lane, seq, abort_flag, pend, npend);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
        if (!ok) break;
        continue;
      }
      if constexpr (COMM == 3 || COMM == 4) {
        const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
        if constexpr (COMM == 3) {
          epilogue_tile_geglu_fwd<BN, C_::kEpiWarps>(p, c, &tmc, tacc, row0, tn, half, bufs, lane, seq);
        } else {
          epilogue_tile_geglu_bwd<BN>(p, c, &tmc, tacc + half * kCols, row0, tn * BN + half * kCols, bufs, lane,
                                      seq);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
        continue;
      }
      epilogue_tile<kCols>(p, &tmc, tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN + half * kCols,
                           row0, tn * BN + half * kCols, bi, alpha, f32_out, bufs, lane, seq);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
    }
    if constexpr (COMM == 2) rs_flush(c, pend, npend, lane);
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  // neither CTA releases its tensor memory or shared memory while the pair's MMAs may still use it
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C_::kTmemCols);
  }
}

template <int BN, bool A_MN, bool B_MN, int COMM = 0>
void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const Params& p, int sms,
                 cudaStream_t stream, const CommParams& comm = CommParams{}) {
  using C_ = Cfg2<BN, pair_epi_warps<COMM>()>;
  auto kern = gemm_pair_kernel<BN, A_MN, B_MN, COMM>;
  static bool configured[64] = {};
  int dev = 0;
  MINT_CUDA_CHECK(cudaGetDevice(&dev));
  if (!configured[dev & 63]) {
    check_smem_optin(C_::kSmemBytes, dev, "gemm");
    MINT_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::kSmemBytes));
    configured[dev & 63] = true;
  }
  const long long tiles = static_cast<long long>((p.M + 255) / 256) * p.tiles_n * p.splits * p.batch;
  const int pairs = static_cast<int>(std::min<long long>(tiles, sms / 2));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(pair_threads<BN, COMM>(), 1, 1);
  cfg.dynamicSmemBytes = C_::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MINT_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, p, comm));
  count_launch();
}

}  // namespace gemm

// C = alpha * op(A) @ op(B) + beta * D.  a_kmajor: A stored [M,K]; else [K,M].  b_kmajor: B stored [N,K]; else [K,N].
// Operands are 2-D, or 3-D [batch, rows, cols] for `batch` independent GEMMs of one shape (every
// 3-D operand needs unit inner stride; the batch stride is free). accumulate = true: C (fp32) +=
// alpha * op(A) @ op(B) through TMA reduce-adds; the contraction is split across CTAs (split-K) when
// the output alone has too few tiles to fill the GPU.
void gemm_bf16(const at::Tensor& A_, const at::Tensor& B_, at::Tensor& C_, const c10::optional<at::Tensor>& D_,
               bool a_kmajor, bool b_kmajor, double alpha, double beta, const c10::optional<at::Tensor>& alpha_t,
               bool accumulate) {
  // MINT_TRACE_GEMM=1: one stderr line per stage of this host function (diagnosing host-side crashes)
  static const bool trace = std::getenv("MINT_TRACE_GEMM") != nullptr;
  if (trace) {
    std::fprintf(stderr, "[gemm] enter A=%p %s B=%p %s C=%p %s dev=%d alpha_t=%d acc=%d\n", A_.data_ptr(),
                 c10::str(A_.sizes()).c_str(), B_.data_ptr(), c10::str(B_.sizes()).c_str(), C_.data_ptr(),
                 c10::str(C_.sizes()).c_str(), A_.is_cuda() ? A_.get_device() : -1,
                 alpha_t.has_value() && alpha_t->defined() ? 1 : 0, accumulate ? 1 : 0);
    std::fflush(stderr);
  }
  check_cuda(A_, "A");
  check_cuda(B_, "B");
  check_cuda(C_, "C");
  MINT_CHECK(A_.dim() == B_.dim() && A_.dim() == C_.dim() && (A_.dim() == 2 || A_.dim() == 3),
             "gemm expects 2-D operands or 3-D batched operands");
  const bool batched = A_.dim() == 3;
  const at::Tensor A = batched ? A_ : A_.unsqueeze(0);
  const at::Tensor B = batched ? B_ : B_.unsqueeze(0);
  at::Tensor C = batched ? C_ : C_.unsqueeze(0);
  const int64_t nb = A.size(0);
  MINT_CHECK(B.size(0) == nb && C.size(0) == nb, "gemm batch sizes differ");
  MINT_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm operands must be bf16");
  MINT_CHECK(A.stride(2) == 1 && B.stride(2) == 1 && C.stride(2) == 1, "gemm operands need unit inner stride");
  MINT_CHECK(C.scalar_type() == at::kBFloat16 || C.scalar_type() == at::kFloat, "C must be bf16 or fp32");
  const int64_t M = a_kmajor ? A.size(1) : A.size(2);
  const int64_t K = a_kmajor ? A.size(2) : A.size(1);
  const int64_t N = b_kmajor ? B.size(1) : B.size(2);
  const int64_t KB = b_kmajor ? B.size(2) : B.size(1);
  MINT_CHECK(K == KB, "gemm K mismatch ", K, " vs ", KB);
  MINT_CHECK(C.size(1) == M && C.size(2) == N, "C has shape ", C_.sizes(), ", expected [", M, ", ", N, "]");
  const int cal = C.scalar_type() == at::kFloat ? 4 : 8;
  MINT_CHECK(C.stride(1) % cal == 0 && (nb == 1 || C.stride(0) % cal == 0), "C strides must be 16-byte aligned");
  MINT_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31) && nb < 65536, "gemm dims too large");
  c10::cuda::CUDAGuard guard(A.device());
  const int dev = A.get_device();
  auto stream = at::cuda::getCurrentCUDAStream();

  gemm::Params p{};
  p.C = C.data_ptr();
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.ldc = C.stride(1);
  p.alpha = static_cast<float>(alpha);
  p.beta = static_cast<float>(beta);
  p.c_fp32 = C.scalar_type() == at::kFloat;
  p.batch = static_cast<int>(nb);
  static const int diag = [] {
    const char* e = std::getenv("MINT_GEMM_DIAG");
    return e == nullptr ? 0 : std::atoi(e);
  }();
  p.diag = diag;
  p.status = status_ptr(dev);
  if (D_.has_value() && D_->defined() && beta != 0.0) {
    const at::Tensor D = batched ? *D_ : D_->unsqueeze(0);
    check_cuda(D, "D");
    MINT_CHECK(D.dim() == 3 && D.size(0) == nb && D.size(1) == M && D.size(2) == N && D.stride(2) == 1,
               "D must match C");
    MINT_CHECK(D.scalar_type() == at::kFloat || D.scalar_type() == at::kBFloat16, "D must be bf16 or fp32");
    MINT_CHECK(D.stride(1) % (D.scalar_type() == at::kFloat ? 4 : 8) == 0, "D row stride must be 16-byte aligned");
    p.D = D.data_ptr();
    p.ldd = D.stride(1);
    p.sd = D.stride(0);
    p.d_fp32 = D.scalar_type() == at::kFloat;
  }
  if (alpha_t.has_value() && alpha_t->defined()) {
    MINT_CHECK(alpha_t->scalar_type() == at::kFloat && alpha_t->numel() == 1 && alpha_t->is_cuda(),
               "alpha tensor must be a 1-element fp32 CUDA tensor");
    p.alpha_ptr = alpha_t->data_ptr<float>();
  }
  if (M == 0 || N == 0 || nb == 0) return;
  if (K == 0) {
    // empty contraction: C = beta * D
    if (p.D != nullptr) {
      C_.copy_(D_->to(C_.scalar_type()).mul(beta));
    } else if (!accumulate) {
      C_.zero_();
    }
    return;
  }
  const int sms = num_sms(dev);
  const int kblocks = static_cast<int>((K + gemm::BK - 1) / gemm::BK);
  // CTA pairs (256-row tiles on 2 SMs) when their work items -- tiles, times the split-K factor an
  // accumulating GEMM may add -- fill at least 90% of the pairs; MINT_GEMM_PAIR=0 disables them
  static const bool pair_enabled = [] {
    const char* e = std::getenv("MINT_GEMM_PAIR");
    return e == nullptr || e[0] != '0';
  }();
  const int pairs = sms / 2;
  const int64_t pair_tiles = nb * ((M + 255) / 256) * ((N + 255) / 256);
  // split-K factor of an accumulating GEMM: the smallest that fills >= 90% of every wave of workers
  // (each split keeps >= 4 k-blocks)
  auto pick_splits = [&](int64_t tiles, int workers) -> int {
    if (tiles >= workers || kblocks < 8) return 1;
    const int64_t max_s = std::max<int64_t>(1, kblocks / 4);
    for (int64_t sp = 1; sp <= max_s; ++sp) {
      const int64_t items = tiles * sp;
      const int64_t waves = (items + workers - 1) / workers;
      if (items * 10 >= waves * workers * 9) return static_cast<int>(sp);
    }
    return static_cast<int>(std::min<int64_t>(max_s, (workers + tiles - 1) / tiles));
  };
  const int pair_splits = accumulate ? pick_splits(pair_tiles, pairs) : 1;
  const bool use_pair = pair_enabled && M >= 256 && N > 128 && pair_tiles * pair_splits * 10 >= pairs * 9;
  int BN = 256;
  if (!use_pair) {
    const int64_t tiles256 = nb * ((M + 127) / 128) * ((N + 255) / 256);
    BN = (N > 128 && tiles256 >= sms) ? 256 : 128;
  }
  p.tiles_m = static_cast<int>((M + 127) / 128);
  p.tiles_n = static_cast<int>((N + BN - 1) / BN);
  p.splits = 1;
  p.kbps = kblocks;
  if (accumulate) {
    MINT_CHECK(p.c_fp32, "accumulating GEMM needs an fp32 C");
    MINT_CHECK(p.D == nullptr, "accumulating GEMM adds into C; D is not used");
    p.atomic_out = 1;
    int splits = 1;
    if (use_pair) {
      splits = pair_splits;
    } else {
      splits = pick_splits(nb * p.tiles_m * p.tiles_n, sms);
    }
    splits = std::max(splits, 1);
    p.kbps = (kblocks + splits - 1) / splits;
    p.splits = (kblocks + p.kbps - 1) / p.kbps;
  }
  MINT_CHECK(static_cast<int64_t>(p.tiles_m) * p.tiles_n * p.splits * nb < (1ll << 31), "too many GEMM tiles");
  // 3-D maps {inner, outer, batch}; for a single GEMM the batch stride only has to be 16-byte aligned
  auto bstride = [&](const at::Tensor& t) -> uint64_t {
    return nb > 1 ? static_cast<uint64_t>(t.stride(0)) : static_cast<uint64_t>(t.size(1) * t.stride(1));
  };
  const uint64_t lda = A.stride(1), ldb = B.stride(1);
  constexpr int BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  constexpr int SW128 = CU_TENSOR_MAP_SWIZZLE_128B;
  const CUtensorMap ta = a_kmajor ? make_tmap_3d(A.data_ptr(), BF, 2, K, M, nb, lda, bstride(A), 64, 128, 1, SW128)
                                  : make_tmap_3d(A.data_ptr(), BF, 2, M, K, nb, lda, bstride(A), 64, 64, 1, SW128);
  const uint32_t bbox = use_pair ? BN / 2 : BN;  // a CTA of a pair loads half of the B tile
  const CUtensorMap tb = b_kmajor ? make_tmap_3d(B.data_ptr(), BF, 2, K, N, nb, ldb, bstride(B), 64, bbox, 1, SW128)
                                  : make_tmap_3d(B.data_ptr(), BF, 2, N, K, nb, ldb, bstride(B), 64, 64, 1, SW128);
  const bool f32c = p.c_fp32 != 0;
  // store boxes: 32 rows x 128 bytes (32 fp32 or 64 bf16 columns), 128B swizzle
  const CUtensorMap tcm = make_tmap_3d(C.data_ptr(), f32c ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : BF, f32c ? 4 : 2, N, M,
                                       nb, C.stride(1), bstride(C), f32c ? 32 : 64, 32, 1, SW128);
  const bool a_mn = !a_kmajor, b_mn = !b_kmajor;
  if (trace) {
    std::fprintf(stderr, "[gemm] maps ok M=%lld N=%lld K=%lld pair=%d BN=%d splits=%d status=%p\n",
                 static_cast<long long>(M), static_cast<long long>(N), static_cast<long long>(K), use_pair ? 1 : 0, BN,
                 p.splits, static_cast<void*>(p.status));
    std::fflush(stderr);
  }
#define MINT_GEMM_DISPATCH(BNV)                                                       \
  if (!a_mn && !b_mn) gemm::launch<BNV, false, false>(ta, tb, tcm, p, sms, stream);   \
  else if (!a_mn && b_mn) gemm::launch<BNV, false, true>(ta, tb, tcm, p, sms, stream); \
  else if (a_mn && !b_mn) gemm::launch<BNV, true, false>(ta, tb, tcm, p, sms, stream); \
  else gemm::launch<BNV, true, true>(ta, tb, tcm, p, sms, stream);
#define MINT_GEMM_DISPATCH_PAIR(BNV)                                                       \
  if (!a_mn && !b_mn) gemm::launch_pair<BNV, false, false>(ta, tb, tcm, p, sms, stream);   \
  else if (!a_mn && b_mn) gemm::launch_pair<BNV, false, true>(ta, tb, tcm, p, sms, stream); \
  else if (a_mn && !b_mn) gemm::launch_pair<BNV, true, false>(ta, tb, tcm, p, sms, stream); \
  else gemm::launch_pair<BNV, true, true>(ta, tb, tcm, p, sms, stream);
  if (use_pair) {
    MINT_GEMM_DISPATCH_PAIR(256)
  } else if (BN == 256) {
    MINT_GEMM_DISPATCH(256)
  } else {
    MINT_GEMM_DISPATCH(128)
  }
#undef MINT_GEMM_DISPATCH
#undef MINT_GEMM_DISPATCH_PAIR
  if (trace) {
    std::fprintf(stderr, "[gemm] launched\n");
    std::fflush(stderr);
  }
}

namespace {

gemm::Params comm_params_base(const at::Tensor& A, const at::Tensor& B, const at::Tensor& C, bool b_kmajor, int dev,
                              int64_t& M, int64_t& N, int64_t& K) {
  check_contig(A, "A");
  check_cuda(B, "B");
  check_contig(C, "C");
  MINT_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "fused TP GEMM expects 2-D operands");
  MINT_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16 && C.scalar_type() == at::kBFloat16,
             "fused TP GEMM operands must be bf16");
  MINT_CHECK(B.stride(1) == 1, "B needs unit inner stride");
  M = A.size(0);
  K = A.size(1);
  N = b_kmajor ? B.size(0) : B.size(1);
  MINT_CHECK((b_kmajor ? B.size(1) : B.size(0)) == K, "fused TP GEMM K mismatch");
  MINT_CHECK((K * 2) % 16 == 0 && (N * 2) % 16 == 0, "fused TP GEMM needs K and N multiples of 8");
  gemm::Params p{};
  p.C = C.data_ptr();
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.ldc = C.stride(0);
  p.alpha = 1.f;
  p.batch = 1;
  p.splits = 1;
  p.tiles_m = static_cast<int>((M + 127) / 128);
  p.tiles_n = static_cast<int>((N + 255) / 256);
  p.kbps = static_cast<int>((K + gemm::BK - 1) / gemm::BK);
  p.status = status_ptr(dev);
  return p;
}

gemm::CommParams comm_common(int64_t rank, int64_t world, int64_t seg, int64_t seq, int64_t M, const at::Tensor& arrive,
                             const std::vector<int64_t>& arrive_peers) {
  MINT_CHECK(world >= 2 && world <= 8 && rank >= 0 && rank < world, "fused TP needs 2..8 ranks");
  MINT_CHECK(seg % 256 == 0 && M % (seg * world) == 0, "fused TP needs segments of a multiple of 256 rows and M a ",
             "multiple of segment x world (M=", M, " seg=", seg, " world=", world, ")");
  MINT_CHECK(static_cast<int64_t>(arrive_peers.size()) == world, "one arrive pointer per rank");
  check_contig(arrive, "arrive");
  MINT_CHECK(arrive.scalar_type() == at::kInt && arrive.numel() >= world, "arrive must be int32 [world]");
  gemm::CommParams c{};
  c.rank = static_cast<int>(rank);
  c.world = static_cast<int>(world);
  c.seg = static_cast<int>(seg);
  c.seq = static_cast<int>(seq);
  c.mc = M / world;
  c.arrive_local = arrive.data_ptr<int>();
  for (int q = 0; q < world; ++q) c.arrive_peer[q] = reinterpret_cast<int*>(arrive_peers[q]);
  return c;
}

}  // namespace

// GeGLU MLP halves with the activation fused into the GEMM epilogues (CTA-pair kernel, BN 256).
//   forward:  X [M, K] @ W12^T, W12 = [fc1; fc2] as one [2F, K] bf16 matrix -> AB [M, 2F] (a | b,
//             kept for the backward) and H = gelu_tanh(a) * b [M, F]
//   backward: dh = DY [M, D] @ W3 (W3 [D, F], the fc3 weight) never stored; DAB [M, 2F] =
//             [dh * b * gelu'(a) | dh * gelu(a)] from AB
void gemm_geglu_fwd(const at::Tensor& X, const at::Tensor& W12, at::Tensor& AB, at::Tensor& H) {
  c10::cuda::CUDAGuard guard(X.device());
  const int dev = X.get_device();
  int64_t M, N2, K;
  gemm::Params p = comm_params_base(X, W12, AB, true, dev, M, N2, K);
  const int64_t F = N2 / 2;
  MINT_CHECK(N2 % 256 == 0, "GeGLU GEMM needs the hidden width F a multiple of 128");
  check_contig(H, "H");
  MINT_CHECK(H.scalar_type() == at::kBFloat16 && H.dim() == 2 && H.size(0) == M && H.size(1) == F,
             "H must be bf16 [M, F]");
  MINT_CHECK(AB.size(0) == M && AB.size(1) == N2, "AB must be bf16 [M, 2F]");
  if (M == 0) return;
  gemm::CommParams c{};
  c.geglu_f = static_cast<int>(F);
  constexpr int BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  constexpr int SW128 = CU_TENSOR_MAP_SWIZZLE_128B;
  c.geglu_map = make_tmap_3d(H.data_ptr(), BF, 2, F, M, 1, F, M * F, 64, 32, 1, SW128);
  const CUtensorMap ta = make_tmap_3d(X.data_ptr(), BF, 2, K, M, 1, X.stride(0), M * X.stride(0), 64, 128, 1, SW128);
  const uint64_t ldb = W12.stride(0);
  const CUtensorMap tb = make_tmap_3d(W12.data_ptr(), BF, 2, K, N2, 1, ldb, N2 * ldb, 64, 128, 1, SW128);
  const CUtensorMap tc = make_tmap_3d(AB.data_ptr(), BF, 2, N2, M, 1, N2, M * N2, 64, 32, 1, SW128);
  gemm::launch_pair<256, false, false, 3>(ta, tb, tc, p, num_sms(dev), at::cuda::getCurrentCUDAStream(), c);
}

void gemm_geglu_bwd(const at::Tensor& DY, const at::Tensor& W3, const at::Tensor& AB, at::Tensor& DAB) {
  c10::cuda::CUDAGuard guard(DY.device());
  const int dev = DY.get_device();
  int64_t M, F, K;
  gemm::Params p = comm_params_base(DY, W3, DAB, false, dev, M, F, K);  // N = F (dh columns)
  MINT_CHECK(F % 128 == 0, "GeGLU GEMM needs the hidden width F a multiple of 128");
  check_contig(AB, "AB");
  MINT_CHECK(AB.scalar_type() == at::kBFloat16 && AB.dim() == 2 && AB.size(0) == M && AB.size(1) == 2 * F,
             "AB must be bf16 [M, 2F]");
  MINT_CHECK(DAB.size(0) == M && DAB.size(1) == 2 * F, "DAB must be bf16 [M, 2F]");
  if (M == 0) return;
  p.N = static_cast<int>(F);
  p.ldc = 2 * F;
  p.tiles_n = static_cast<int>((F + 255) / 256);
  gemm::CommParams c{};
  c.geglu_f = static_cast<int>(F);
  c.geglu_ab = reinterpret_cast<const __nv_bfloat16*>(AB.data_ptr());
  constexpr int BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  constexpr int SW128 = CU_TENSOR_MAP_SWIZZLE_128B;
  const CUtensorMap ta = make_tmap_3d(DY.data_ptr(), BF, 2, K, M, 1, DY.stride(0), M * DY.stride(0), 64, 128, 1, SW128);
  const uint64_t ldb = W3.stride(0);
  const CUtensorMap tb = make_tmap_3d(W3.data_ptr(), BF, 2, F, K, 1, ldb, K * ldb, 64, 64, 1, SW128);
  const CUtensorMap tc = make_tmap_3d(DAB.data_ptr(), BF, 2, 2 * F, M, 1, 2 * F, M * 2 * F, 64, 32, 1, SW128);
  gemm::launch_pair<256, false, true, 4>(ta, tb, tc, p, num_sms(dev), at::cuda::getCurrentCUDAStream(), c);
}

// C[M, N] = A[M, K] @ op(B) with the all-gather of A's rows over the tensor-parallel group fused in:
// A is this rank's symmetric gathered buffer holding its own chunk; `src_ptrs[p]` is rank p's
// gathered buffer (the same layout), from which this kernel pulls rank p's chunk over NVLink.
void gemm_ag(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool b_kmajor, const std::vector<int64_t>& src_ptrs,
             const at::Tensor& arrive, const std::vector<int64_t>& arrive_peers, at::Tensor& rowflag, at::Tensor& claim,
             int64_t rank, int64_t world, int64_t seg, int64_t seq) {
  c10::cuda::CUDAGuard guard(A.device());
  const int dev = A.get_device();
  auto stream = at::cuda::getCurrentCUDAStream();
  int64_t M, N, K;
  gemm::Params p = comm_params_base(A, B, C, b_kmajor, dev, M, N, K);
  MINT_CHECK(C.size(0) == M && C.size(1) == N, "C must be [M, N]");
  gemm::CommParams c = comm_common(rank, world, seg, seq, M, arrive, arrive_peers);
  MINT_CHECK(static_cast<int64_t>(src_ptrs.size()) == world, "one source pointer per rank");
  for (int q = 0; q < world; ++q) c.ag_src[q] = reinterpret_cast<const uint8_t*>(src_ptrs[q]);
  c.ag_dst = static_cast<uint8_t*>(A.data_ptr());
  c.ag_row_bytes = K * 2;
  check_contig(rowflag, "rowflag");
  MINT_CHECK(rowflag.scalar_type() == at::kInt && rowflag.numel() >= M / 128, "rowflag must be int32 [M / 128]");
  check_contig(claim, "claim");
  MINT_CHECK(claim.scalar_type() == at::kLong && claim.numel() >= 1, "claim must be int64 [1]");
  c.rowflag = rowflag.data_ptr<int>();
  c.blockcnt = rowflag.data_ptr<int>() + rowflag.numel() / 2;  // second half of the flag tensor
  MINT_CHECK(rowflag.numel() / 2 >= M / 128, "rowflag must hold 2 x M / 128 int32 (flags, piece counters)");
  c.claim = reinterpret_cast<unsigned long long*>(claim.data_ptr<int64_t>());
  MINT_CUDA_CHECK(cudaMemsetAsync(c.claim, 0, sizeof(unsigned long long), stream));
  constexpr int BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  constexpr int SW128 = CU_TENSOR_MAP_SWIZZLE_128B;
  const CUtensorMap ta = make_tmap_3d(A.data_ptr(), BF, 2, K, M, 1, K, M * K, 64, 128, 1, SW128);
  const uint64_t ldb = B.stride(0);
  const CUtensorMap tb = b_kmajor ? make_tmap_3d(B.data_ptr(), BF, 2, K, N, 1, ldb, N * ldb, 64, 128, 1, SW128)
                                  : make_tmap_3d(B.data_ptr(), BF, 2, N, K, 1, ldb, K * ldb, 64, 64, 1, SW128);
  const CUtensorMap tc = make_tmap_3d(C.data_ptr(), BF, 2, N, M, 1, C.stride(0), M * C.stride(0), 64, 32, 1, SW128);
  const int sms = num_sms(dev);
  if (b_kmajor) {
    gemm::launch_pair<256, false, false, 1>(ta, tb, tc, p, sms, stream, c);
  } else {
    gemm::launch_pair<256, false, true, 1>(ta, tb, tc, p, sms, stream, c);
  }
}

// out[M / world, N] = this rank's chunk of sum over the group of (A[M, K] @ op(B)): the GEMM with
// the reduce-scatter of its output rows fused in. `push_ptrs[p]` is rank p's receive slot for this
// rank ([M / world, N] bf16), `flag_ptrs[p]` rank p's flag block for this rank; `recv` / `flags` are
// this rank's own receive slots [world, M / world, N] and flag blocks [world, stride].
void gemm_rs(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, bool b_kmajor,
             const std::vector<int64_t>& push_ptrs, const at::Tensor& recv, const std::vector<int64_t>& flag_ptrs,
             const at::Tensor& flags, const at::Tensor& arrive, const std::vector<int64_t>& arrive_peers, int64_t rank,
             int64_t world, int64_t seg, int64_t seq) {
  c10::cuda::CUDAGuard guard(A.device());
  const int dev = A.get_device();
  auto stream = at::cuda::getCurrentCUDAStream();
  int64_t M, N, K;
  gemm::Params p = comm_params_base(A, B, out, b_kmajor, dev, M, N, K);
  gemm::CommParams c = comm_common(rank, world, seg, seq, M, arrive, arrive_peers);
  MINT_CHECK(out.size(0) == c.mc && out.size(1) == N && out.stride(0) == N, "out must be contiguous [M / world, N]");
  check_contig(recv, "recv");
  MINT_CHECK(recv.scalar_type() == at::kBFloat16 && recv.numel() >= world * c.mc * N, "recv must be bf16 [world, Mc, N]");
  check_contig(flags, "flags");
  const int64_t tiles_n = (N + 255) / 256;
  MINT_CHECK(flags.scalar_type() == at::kInt && flags.dim() == 2 && flags.size(0) == world &&
                 flags.size(1) >= (c.mc / 128) * tiles_n * 4,
             "flags must be int32 [world, >= Mc / 128 * tiles_n * 4]");
  c.rs_flag_stride = flags.size(1);
  MINT_CHECK(static_cast<int64_t>(push_ptrs.size()) == world && static_cast<int64_t>(flag_ptrs.size()) == world,
             "one push / flag pointer per rank");
  constexpr int BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  constexpr int SW128 = CU_TENSOR_MAP_SWIZZLE_128B;
  for (int q = 0; q < world; ++q) {
    c.rs_push[q] = reinterpret_cast<__nv_bfloat16*>(push_ptrs[q]);
    c.rs_flag_peer[q] = reinterpret_cast<int*>(flag_ptrs[q]);
    // peer q's receive slot for this rank, [Mc, N] bf16 in its symmetric buffer: the epilogue's
    // 32 x 64 staging boxes leave through TMA stores with this map (plain stores, no multicast)
    if (q != rank) {
      c.rs_push_map[q] = make_tmap_3d(c.rs_push[q], BF, 2, N, c.mc, 1, N, c.mc * N, 64, 32, 1, SW128);
    }
  }
  // MINT_RS_LAG: how many 256-row tiles this rank's own tile k trails the peers' tile k (default 8)
  static const int rs_lag = [] {
    const char* e = std::getenv("MINT_RS_LAG");
    return e == nullptr ? 8 : std::max(1, std::atoi(e));
  }();
  c.rs_lag = rs_lag;
  c.rs_recv = reinterpret_cast<const __nv_bfloat16*>(recv.data_ptr());
  c.rs_flag_local = flags.data_ptr<int>();
  const CUtensorMap ta = make_tmap_3d(A.data_ptr(), BF, 2, K, M, 1, A.stride(0), M * A.stride(0), 64, 128, 1, SW128);
  const uint64_t ldb = B.stride(0);
  const CUtensorMap tb = b_kmajor ? make_tmap_3d(B.data_ptr(), BF, 2, K, N, 1, ldb, N * ldb, 64, 128, 1, SW128)
                                  : make_tmap_3d(B.data_ptr(), BF, 2, N, K, 1, ldb, K * ldb, 64, 64, 1, SW128);
  const CUtensorMap tc = make_tmap_3d(out.data_ptr(), BF, 2, N, c.mc, 1, N, c.mc * N, 64, 32, 1, SW128);
  const int sms = num_sms(dev);
  if (b_kmajor) {
    gemm::launch_pair<256, false, false, 2>(ta, tb, tc, p, sms, stream, c);
  } else {
    gemm::launch_pair<256, false, true, 2>(ta, tb, tc, p, sms, stream, c);
  }
}

}  // namespace mint
