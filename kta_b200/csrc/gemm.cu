// 16-bit GEMM on the 5th-generation tensor cores (tcgen05), sm_100a.
//
//   C[M,N] = A[M,K] . op(B),  op(B) = B[N,K]^T ("tn", K-major B)  or  B[K,N] ("nn").
//
// It replaces KTA's TileLang hgemm (perfmodel/testset/gen.py:255-303) and the seed GEMM
// family (knowledge/seed/families/gemm_fp16_tilelang/gen.py:32-112): same contraction,
// fp32 accumulation, 16-bit output. The design is B200-first, not a translation:
//
//   * persistent grid of one CTA per SM walking a grouped raster of 128 x BN output tiles;
//   * warp 0: TMA producer (128-byte swizzled K-major tiles into a STAGES-deep mbarrier
//     ring); warp 1: TMEM allocator and the single-thread tcgen05.mma issuer;
//     warps 2-5: epilogue (tcgen05.ld -> bf16/f16 -> swizzled smem -> TMA store);
//   * the fp32 accumulator lives in TMEM, double buffered (2 x BN columns), so the
//     epilogue of tile i overlaps the main loop of tile i+1;
//   * every mbarrier wait is bounded (kta_common.cuh), no spin can hang the GPU.
//
// Skinny shapes (M <= 64, e.g. the decode-time M = 16) are HBM-bound on B: they run a
// swap-AB kernel (D^T = B . A^T, UMMA M = 128 rows of B, N = M rounded up to 16) split
// along K over a thread-block cluster whose partial sums are reduced through distributed
// shared memory, so every SM streams B and no global workspace is needed.
#include <algorithm>
#include <cstdlib>

#include "kta_common.cuh"
#include "kta_host.h"

namespace kta {
namespace gemm {

constexpr int BM = 128;         // UMMA M (rows of A per tile)
constexpr int BK = 64;          // 16-bit K elements per stage = one 128-byte swizzle row
constexpr int UMMA_K = 16;      // K per tcgen05.mma of kind::f16
constexpr int EPI_WARPS = 4;    // one per TMEM lane quarter
constexpr int NUM_THREADS = 64 + EPI_WARPS * 32;
constexpr int EPI_COLS = 64;    // output columns per staged chunk (128 B of 16-bit values)
constexpr int GROUP_M = 16;     // raster group height (tiles) for L2 reuse

// Watchdog sites (kta_device_status word 1).
enum : unsigned int {
  SITE_PRODUCER_EMPTY = 0x101,
  SITE_MMA_FULL = 0x102,
  SITE_MMA_TEMPTY = 0x103,
  SITE_EPI_TFULL = 0x104,
  SITE_SKINNY_FULL = 0x111,
  SITE_SKINNY_EMPTY = 0x112,
  SITE_SKINNY_TFULL = 0x113,
};

template <int BN, int STAGES>
struct Layout {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int C_BYTES = 32 * EPI_COLS * 2;  // one warp's staged chunk
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_C = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_BAR = OFF_C + EPI_WARPS * 2 * C_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 4;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int TOTAL = OFF_MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;  // slack to align the base to 1024 B
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static_assert(ALLOC <= 232448, "shared memory budget of one sm_100 CTA");
};

// Tile `tile` of a grouped raster: bands of `group_m` tile rows, each band walked column by
// column (a column's group_m tiles are consecutive), so the tiles in flight share a band of
// A panels and a few B panels.
__device__ __forceinline__ void tile_coords_g(int tile, int tiles_m, int tiles_n, int group_m,
                                              int& mb, int& nb) {
  const int per_group = group_m * tiles_n;
  const int group = tile / per_group;
  const int first_m = group * group_m;
  const int gsz = min(tiles_m - first_m, group_m);
  const int r = tile - group * per_group;
  mb = first_m + r % gsz;
  nb = r / gsz;
}

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& mb,
                                            int& nb) {
  tile_coords_g(tile, tiles_m, tiles_n, GROUP_M, mb, nb);
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  const uint32_t a = smem_u32(p);
  return p + ((1024u - (a & 1023u)) & 1023u);
}

// B_KMAJOR: B is [N,K] (tn); otherwise B is [K,N] (nn) and is fed as an MN-major operand.
template <int BN, int STAGES, bool BF16, bool B_KMAJOR>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, int M, int N, int K,
                int rows_per_group, unsigned int* status) {
  using L = Layout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], EPI_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_launch_dependents();
  pdl_wait();  // the previous grid's writes (this launch's inputs) are visible from here on

  const int tiles_m = (M + BM - 1) / BM;
  const int tiles_n = (N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (K + BK - 1) / BK;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, tiles_m, tiles_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status, SITE_PRODUCER_EMPTY)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + L::OFF_A + stage * L::A_BYTES;
          uint8_t* sb = smem + L::OFF_B + stage * L::B_BYTES;
          mbar_arrive_expect_tx(&full[stage], L::A_BYTES + L::B_BYTES);
          tma_load_2d(&tmA, &full[stage], sa, kb * BK, mb * BM);
          if constexpr (B_KMAJOR) {
            tma_load_2d(&tmB, &full[stage], sb, kb * BK, nb * BN);
          } else {
            // [K,N] row-major: BN/64 boxes of 64 N x 64 K, each one MN-major swizzle block.
            // Grouped (MoE): B is [E, K, N] and the tile's rows belong to expert
            // (mb * BM) / rows_per_group.
            const int e = rows_per_group > 0 ? (mb * BM) / rows_per_group : -1;
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) {
              if (e < 0) {
                tma_load_2d(&tmB, &full[stage], sb + j * (64 * BK * 2), nb * BN + j * 64, kb * BK);
              } else {
                tma_load_3d(&tmB, &full[stage], sb + j * (64 * BK * 2), nb * BN + j * 64, kb * BK, e);
              }
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t fmt = BF16 ? 1u : 0u;
      constexpr uint32_t idesc = make_idesc(BM, BN, fmt, fmt, 0u, B_KMAJOR ? 0u : 1u);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, status, SITE_MMA_TEMPTY)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, status, SITE_MMA_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + L::OFF_A + stage * L::A_BYTES);
          const uint32_t b0 = smem_u32(smem + L::OFF_B + stage * L::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            const uint64_t ad = sdesc_sw128(a0 + k * UMMA_K * 2, 16, 1024);
            uint64_t bd;
            if constexpr (B_KMAJOR) {
              bd = sdesc_sw128(b0 + k * UMMA_K * 2, 16, 1024);
            } else {
              // K rows are 128 B apart: 16 K rows per MMA; 64-wide N blocks 8 KB apart.
              bd = sdesc_sw128(b0 + k * UMMA_K * 128, 64 * BK * 2, 1024);
            }
            umma_f16(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);  // frees the smem stage once these MMAs completed
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);  // accumulator complete
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> registers -> smem -> TMA store ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    uint8_t* cbuf = smem + L::OFF_C + (warp - 2) * 2 * L::C_BYTES;
    int acc = 0;
    uint32_t acc_phase = 0;
    int buf = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mb, nb;
      tile_coords(tile, tiles_m, tiles_n, mb, nb);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, status, SITE_EPI_TFULL)) break;
      tc_fence_after();
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN / EPI_COLS; ++c) {
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(t_row + c * EPI_COLS, r0);
        tmem_ld_32x32b_x32(t_row + c * EPI_COLS + 32, r1);
        tmem_ld_wait();
        reg_fence(r0);
        reg_fence(r1);
        if (c == BN / EPI_COLS - 1) {
          // Every column of this accumulator is in registers: hand TMEM back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);
        }
        uint32_t p[32];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          p[j] = pack2<BF16>(__uint_as_float(r0[2 * j]), __uint_as_float(r0[2 * j + 1]));
          p[16 + j] = pack2<BF16>(__uint_as_float(r1[2 * j]), __uint_as_float(r1[2 * j + 1]));
        }
        // The store issued from this buffer two chunks ago must have finished reading it.
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        uint8_t* sbuf = cbuf + buf * L::C_BYTES;
        const uint32_t row = smem_u32(sbuf) + static_cast<uint32_t>(lane) * 128u;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          st_shared_v4(row + ((static_cast<uint32_t>(j) ^ (lane & 7u)) << 4), p[4 * j],
                       p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, sbuf, nb * BN + c * EPI_COLS, mb * BM + q * 32);
          bulk_commit_group();
        }
        buf ^= 1;
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------
// 2-SM variant (tn): a cluster of two CTAs computes one 256 x 256 tile with
// tcgen05.mma.cta_group::2. Each CTA loads its own 128 rows of A and 128 rows of B per
// stage (no multicast); the leader (cluster rank 0) issues the MMAs, which read A and B
// from both CTAs' shared memory, and each CTA's TMEM receives its 128 rows x 256 columns.
// Per SM the tensor core reads 8 KB of operands per 256x256x16 step instead of 12 KB
// for the 1-SM 128x256 tile, and L2 serves a third less operand traffic per FLOP.
// ---------------------------------------------------------------------------------------
constexpr int P_BM = 256;   // rows of A per CTA pair (128 per CTA)

// PBN columns per pair tile (256, or 128 for the grouped expert GEMM): PBN / 2 of B per CTA.
template <int PBN>
struct PairLayout {
  static constexpr int STAGES = PBN == 256 ? 6 : 8;
  static constexpr int A_BYTES = 128 * BK * 2;
  static constexpr int B_BYTES = (PBN / 2) * BK * 2;
  static constexpr int C_BYTES = 32 * EPI_COLS * 2;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_C = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_BAR = OFF_C + EPI_WARPS * 2 * C_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 4;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int TOTAL = OFF_MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * PBN;
  static_assert(ALLOC <= 232448, "shared memory budget of one sm_100 CTA");
  static_assert(B_BYTES % 1024 == 0 && OFF_B % 1024 == 0, "swizzled stages on 1 KB boundaries");
};

// B_KMAJOR: B is [N, K] (tn); otherwise [K, N] (nn), or [groups, K, N] with rows_per_group > 0
// (expert GEMM: a tile's 256 rows all belong to expert (mb * 256) / rows_per_group), fed as an
// MN-major operand in 64-column swizzle blocks.
template <bool BF16, bool B_KMAJOR, int PBN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, int M, int N, int K, int group_m,
                     int l2_hint, int rows_per_group, unsigned int* status) {
  using L = PairLayout<PBN>;
  constexpr int P_STAGES = L::STAGES;
  constexpr int P_BN = PBN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);  // leader's counts both CTAs
  uint64_t* empty = full + P_STAGES;                                 // in each CTA
  uint64_t* tfull = empty + P_STAGES;                                // in each CTA
  uint64_t* tempty = tfull + 2;                                      // leader's counts both
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank_u32();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 2 * EPI_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(L::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  pair_sync();  // both CTAs' barriers are initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_launch_dependents();
  pdl_wait();  // the previous grid's writes (this launch's inputs) are visible from here on

  const int tiles_m = (M + P_BM - 1) / P_BM;
  const int tiles_n = (N + P_BN - 1) / P_BN;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (K + BK - 1) / BK;
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // the band's A panels are read again by the next columns' tiles: keep them in L2 ahead
      // of B, whose panels serve only the tiles of one column
      const uint64_t pol_a = l2_policy_evict_last();
      const uint64_t pol_b = l2_policy_evict_first();
      for (int tile = pair; tile < num_tiles && ok; tile += pairs) {
        int mb, nb;
        tile_coords_g(tile, tiles_m, tiles_n, group_m, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status, SITE_PRODUCER_EMPTY)) {
            ok = false;
            break;
          }
          const uint32_t bar0 = peer_addr(&full[stage], 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * (L::A_BYTES + L::B_BYTES));
          uint8_t* da = smem + L::OFF_A + stage * L::A_BYTES;
          uint8_t* db = smem + L::OFF_B + stage * L::B_BYTES;
          const int ya = mb * P_BM + static_cast<int>(rank) * 128;
          const int yb = nb * P_BN + static_cast<int>(rank) * (P_BN / 2);
          if (l2_hint & 1) {
            tma_load_2d_pair_hint(&tmA, bar0, da, kb * BK, ya, pol_a);
          } else {
            tma_load_2d_pair(&tmA, bar0, da, kb * BK, ya);
          }
          if constexpr (B_KMAJOR) {
            if (l2_hint & 2) {
              tma_load_2d_pair_hint(&tmB, bar0, db, kb * BK, yb, pol_b);
            } else {
              tma_load_2d_pair(&tmB, bar0, db, kb * BK, yb);
            }
          } else {
            // [K, N] (or expert e's [K, N]): this CTA's PBN / 2 columns as 64-column blocks
            const int e = rows_per_group > 0 ? (mb * P_BM) / rows_per_group : -1;
#pragma unroll
            for (int j = 0; j < P_BN / 128; ++j) {
              uint8_t* dj = db + j * (64 * BK * 2);
              if (e < 0) {
                tma_load_2d_pair(&tmB, bar0, dj, yb + j * 64, kb * BK);
              } else {
                tma_load_3d_pair(&tmB, bar0, dj, yb + j * 64, kb * BK, e);
              }
            }
          }
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    if (leader && lane == 0) {
      constexpr uint32_t fmt = BF16 ? 1u : 0u;
      constexpr uint32_t idesc = make_idesc(P_BM, P_BN, fmt, fmt, 0u, B_KMAJOR ? 0u : 1u);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += pairs) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, status, SITE_MMA_TEMPTY)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * P_BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, status, SITE_MMA_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + L::OFF_A + stage * L::A_BYTES);
          const uint32_t b0 = smem_u32(smem + L::OFF_B + stage * L::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            // MN-major B: K rows 128 B apart (16 per MMA), 64-column blocks 8 KB apart
            const uint64_t bd = B_KMAJOR ? sdesc_sw128(b0 + k * UMMA_K * 2, 16, 1024)
                                         : sdesc_sw128(b0 + k * UMMA_K * 128, 64 * BK * 2, 1024);
            umma_f16_pair(d_tmem, sdesc_sw128(a0 + k * UMMA_K * 2, 16, 1024), bd, idesc,
                          (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage]);  // frees this stage in both CTAs
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc]);  // each CTA's half of the accumulator is complete
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // ---------------- epilogue (both CTAs): this CTA's 128 rows x 256 columns ----------------
    const int q = warp & 3;
    uint8_t* cbuf = smem + L::OFF_C + (warp - 2) * 2 * L::C_BYTES;
    int acc = 0;
    uint32_t acc_phase = 0;
    int buf = 0;
    const uint32_t tempty0[2] = {peer_addr(&tempty[0], 0), peer_addr(&tempty[1], 0)};
    // C is written once and never read back here: its lines should not push A panels out
    const uint64_t pol_c = l2_policy_evict_first();
    for (int tile = pair; tile < num_tiles; tile += pairs) {
      int mb, nb;
      tile_coords_g(tile, tiles_m, tiles_n, group_m, mb, nb);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, status, SITE_EPI_TFULL)) break;
      tc_fence_after();
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * P_BN);
      const int row0 = mb * P_BM + static_cast<int>(rank) * 128 + q * 32;
#pragma unroll 1
      for (int c = 0; c < P_BN / EPI_COLS; ++c) {
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(t_row + c * EPI_COLS, r0);
        tmem_ld_32x32b_x32(t_row + c * EPI_COLS + 32, r1);
        tmem_ld_wait();
        reg_fence(r0);
        reg_fence(r1);
        if (c == P_BN / EPI_COLS - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(tempty0[acc]);
        }
        uint32_t pk[32];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          pk[j] = pack2<BF16>(__uint_as_float(r0[2 * j]), __uint_as_float(r0[2 * j + 1]));
          pk[16 + j] = pack2<BF16>(__uint_as_float(r1[2 * j]), __uint_as_float(r1[2 * j + 1]));
        }
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        uint8_t* sbuf = cbuf + buf * L::C_BYTES;
        const uint32_t rowa = smem_u32(sbuf) + static_cast<uint32_t>(lane) * 128u;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          st_shared_v4(rowa + ((static_cast<uint32_t>(j) ^ (lane & 7u)) << 4), pk[4 * j],
                       pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (l2_hint & 4) {
            tma_store_2d_hint(&tmC, sbuf, nb * P_BN + c * EPI_COLS, row0, pol_c);
          } else {
            tma_store_2d(&tmC, sbuf, nb * P_BN + c * EPI_COLS, row0);
          }
          bulk_commit_group();
        }
        buf ^= 1;
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  pair_sync();  // the leader's MMAs into this CTA's TMEM and remote arrivals are over
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(L::TMEM_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------------------
// Skinny M (<= 64): swap-AB, K split over a cluster, DSMEM reduction.
// ---------------------------------------------------------------------------------------
constexpr int SK_ROWS = 128;  // rows of B (columns of C) per CTA: UMMA M
constexpr int SK_SUB = 2;     // 64-wide K boxes per stage: each row of B is read in 256-byte runs
constexpr int SK_BK = SK_SUB * BK;
constexpr int SK_THREADS = NUM_THREADS;

template <int MP>
struct SkinnyLayout {
  static constexpr int B_SUB = SK_ROWS * BK * 2;                  // one box: 128 rows of B
  static constexpr int A_SUB = ((MP * BK * 2 + 1023) / 1024) * 1024;  // one box: MP rows of A
  static constexpr int B_BYTES = SK_SUB * B_SUB;                  // "A operand"
  static constexpr int A_BYTES = SK_SUB * A_SUB;                  // "B operand"
  static constexpr int STAGE_BYTES = B_BYTES + A_BYTES;
  // as many stages as fit (6 for M <= 16): the bytes in flight per SM set the bandwidth
  static constexpr int STAGES = (232448 - 2048) / STAGE_BYTES < 6 ? (232448 - 2048) / STAGE_BYTES : 6;
  static constexpr int OFF_STAGE = 0;
  // [cluster-1][128][MP] fp32 partials; reuses the stage ring once every rank's main loop
  // is over (the first cluster barrier of the epilogue).
  static constexpr int OFF_RED = 0;
  static constexpr int RED_SLOT_BYTES = SK_ROWS * MP * 4;
  static constexpr int MAX_CLUSTER = (STAGES * STAGE_BYTES) / RED_SLOT_BYTES + 1;
  static constexpr int OFF_BAR = STAGES * STAGE_BYTES;
  static constexpr int OFF_MISC = OFF_BAR + (2 * STAGES + 1) * 8;
  static constexpr int TOTAL = OFF_MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;
  static constexpr uint32_t TMEM_COLS = MP <= 32 ? 32 : 64;
  static_assert(ALLOC <= 232448, "shared memory budget of one sm_100 CTA");
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n"
               "barrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

template <int MP, bool BF16>
__global__ void __launch_bounds__(SK_THREADS, 1)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmB, void* __restrict__ Cv, int M,
                       int N, int K, int64_t ldc, int csize, unsigned int* status) {
  using L = SkinnyLayout<MP>;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + L::STAGES;
  uint64_t* tfull = empty + L::STAGES;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  float* red = reinterpret_cast<float*>(smem + L::OFF_RED);

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int tile = blockIdx.x / csize;
  const int num_kb = (K + SK_BK - 1) / SK_BK;
  const int kb_begin = static_cast<int>((static_cast<int64_t>(rank) * num_kb) / csize);
  const int kb_end = static_cast<int>((static_cast<int64_t>(rank + 1) * num_kb) / csize);

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // every CTA of the cluster runs before any DSMEM access
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_launch_dependents();
  pdl_wait();  // the previous grid's writes (this launch's inputs) are visible from here on

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status, SITE_SKINNY_EMPTY)) break;
        uint8_t* st = smem + L::OFF_STAGE + stage * L::STAGE_BYTES;
        // expect the full boxes: out-of-range parts are zero-filled and still counted
        mbar_arrive_expect_tx(&full[stage], SK_SUB * (L::B_SUB + MP * BK * 2));
#pragma unroll
        for (int u = 0; u < SK_SUB; ++u) {
          tma_load_2d(&tmB, &full[stage], st + u * L::B_SUB, kb * SK_BK + u * BK, tile * SK_ROWS);
        }
#pragma unroll
        for (int u = 0; u < SK_SUB; ++u) {
          tma_load_2d(&tmA, &full[stage], st + L::B_BYTES + u * L::A_SUB, kb * SK_BK + u * BK, 0);
        }
        if (++stage == L::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t fmt = BF16 ? 1u : 0u;
      constexpr uint32_t idesc = make_idesc(SK_ROWS, MP, fmt, fmt, 0u, 0u);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag, status, SITE_SKINNY_FULL)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t s0 = smem_u32(smem + L::OFF_STAGE + stage * L::STAGE_BYTES);
#pragma unroll
        for (int k = 0; k < SK_BK / UMMA_K; ++k) {
          const int u = k / (BK / UMMA_K), kk = k % (BK / UMMA_K);
          const uint64_t ad = sdesc_sw128(s0 + u * L::B_SUB + kk * UMMA_K * 2, 16, 1024);
          const uint64_t bd =
              sdesc_sw128(s0 + L::B_BYTES + u * L::A_SUB + kk * UMMA_K * 2, 16, 1024);
          umma_f16(tmem_base, ad, bd, idesc, (kb > kb_begin || k > 0) ? 1u : 0u);
        }
        umma_commit(&empty[stage]);
        if (++stage == L::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) umma_commit(tfull);
    }
  }

  // Epilogue warps (2-5) read the partial D^T tile: lane = row of B (column of C).
  float acc[MP];
  const bool epi = warp >= 2;
  const int q = warp & 3;
  const int row = q * 32 + lane;  // 0..127 within the tile
  bool have = false;
  if (epi) {
    if (kb_end > kb_begin) {
      if (mbar_wait(tfull, 0, abort_flag, status, SITE_SKINNY_TFULL)) {
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll
        for (int c = 0; c < MP; c += 16) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(taddr + c, r);
          tmem_ld_wait();
          reg_fence(r);
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[c + j] = __uint_as_float(r[j]);
        }
        have = true;
      }
    }
    if (!have) {
#pragma unroll
      for (int j = 0; j < MP; ++j) acc[j] = 0.f;
    }
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // every rank's main loop is over: the stage rings are free
  if (epi && rank != 0) {
    // Send the partial to rank 0's reduction slot [rank-1][row][MP].
    const uint32_t local = smem_u32(red + ((rank - 1) * SK_ROWS + row) * MP);
    const uint32_t remote = map_to_rank(local, 0);
#pragma unroll
    for (int j = 0; j < MP; ++j) st_cluster_f32(remote + j * 4, acc[j]);
  }
  __syncwarp();
  cluster_sync_all();  // partials of every rank are in rank 0's shared memory
  if (epi && rank == 0) {
    for (int r = 1; r < csize; ++r) {
      const float* src = red + ((r - 1) * SK_ROWS + row) * MP;
#pragma unroll
      for (int j = 0; j < MP; ++j) acc[j] += src[j];
    }
    const int n = tile * SK_ROWS + row;
    if (n < N) {
      T* C = reinterpret_cast<T*>(Cv);
#pragma unroll
      for (int j = 0; j < MP; ++j) {
        if (j < M) {
          if constexpr (BF16) {
            C[static_cast<int64_t>(j) * ldc + n] = __float2bfloat16_rn(acc[j]);
          } else {
            C[static_cast<int64_t>(j) * ldc + n] = __float2half_rn(acc[j]);
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------
template <typename Kern>
int set_smem(Kern kernel, int bytes) {
  return set_kernel_smem(reinterpret_cast<const void*>(kernel), bytes);
}

// groups > 0 (MoE, B [K, N] layout only): B is [groups, K, N] and rows
// [g * M / groups, (g + 1) * M / groups) of A and C use B[g].
template <int BN, int STAGES, bool BF16, bool B_KMAJOR>
int launch_main(const void* A, const void* B, void* C, int M, int N, int K, int64_t lda,
                int64_t ldb, int64_t ldc, cudaStream_t stream, int groups = 0) {
  using L = Layout<BN, STAGES>;
  const CUtensorMapDataType dt =
      BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb, tc;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(lda) * 2};
    const uint32_t box[2] = {BK, BM};
    int s = encode_tmap(&ta, dt, 2, A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  if (B_KMAJOR) {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldb) * 2};
    const uint32_t box[2] = {BK, BN};
    int s = encode_tmap(&tb, dt, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  } else if (groups > 0) {
    const uint64_t dims[3] = {static_cast<uint64_t>(N), static_cast<uint64_t>(K),
                              static_cast<uint64_t>(groups)};
    const uint64_t strides[2] = {static_cast<uint64_t>(ldb) * 2,
                                 static_cast<uint64_t>(ldb) * 2 * static_cast<uint64_t>(K)};
    const uint32_t box[3] = {64, BK, 1};
    int s = encode_tmap(&tb, dt, 3, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  } else {
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(K)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldb) * 2};
    const uint32_t box[2] = {64, BK};
    int s = encode_tmap(&tb, dt, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldc) * 2};
    const uint32_t box[2] = {EPI_COLS, 32};
    int s = encode_tmap(&tc, dt, 2, C, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  auto kernel = gemm_kernel<BN, STAGES, BF16, B_KMAJOR>;
  int s = set_smem(kernel, L::ALLOC);
  if (s != KTA_OK) return s;
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int sms = current_sm_count();
  const int grid = std::max(1, std::min(tiles, sms));
  const int rows_per_group = groups > 0 ? M / groups : 0;
  return launch_ex(kernel, dim3(grid), dim3(NUM_THREADS), L::ALLOC, stream, 1, ta, tb, tc, M, N,
                   K, rows_per_group, device_status_ptr());
}

template <int MP, bool BF16>
int launch_skinny(const void* A, const void* B, void* C, int M, int N, int K, int64_t lda,
                  int64_t ldb, int64_t ldc, cudaStream_t stream) {
  using L = SkinnyLayout<MP>;
  const CUtensorMapDataType dt =
      BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(lda) * 2};
    const uint32_t box[2] = {BK, static_cast<uint32_t>(MP)};
    int s = encode_tmap(&ta, dt, 2, A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldb) * 2};
    const uint32_t box[2] = {BK, SK_ROWS};
    int s = encode_tmap(&tb, dt, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  auto kernel = gemm_skinny_kernel<MP, BF16>;
  int s = set_smem(kernel, L::ALLOC);
  if (s != KTA_OK) return s;
  const int tiles = (N + SK_ROWS - 1) / SK_ROWS;
  const int num_kb = (K + SK_BK - 1) / SK_BK;
  const int sms = current_sm_count();
  // Cluster size: the largest power of two (<= 8) that keeps tiles x size within one wave
  // and leaves every rank at least two k-blocks.
  int cs = 1;
  while (cs < 8 && cs * 2 <= L::MAX_CLUSTER && tiles * cs * 2 <= sms && num_kb >= cs * 4) {
    cs *= 2;
  }

  void* Cp = C;
  return launch_ex(kernel, dim3(static_cast<unsigned>(tiles * cs)), dim3(SK_THREADS), L::ALLOC,
                   stream, static_cast<unsigned>(cs), ta, tb, Cp, M, N, K, ldc, cs,
                   device_status_ptr());
}

// Raster of the pair kernel: bands of P_GROUP_M tile rows (8 x 256 rows: a 32 MB band of A
// for K = 8192, which stays in L2 under the evict-last policy while B streams past it);
// KTA_GEMM_GROUP=<n> and KTA_GEMM_L2HINT=<bits> override both (tuning runs; bit 0: A
// loads evict-last, bit 1: B loads evict-first, bit 2: C stores evict-first).
constexpr int P_GROUP_M = 8;
inline void pair_raster_env(int& group_m, int& l2_hint) {
  if (const char* g = std::getenv("KTA_GEMM_GROUP")) {
    const int v = std::atoi(g);
    if (v >= 1 && v <= 64) group_m = v;
  }
  if (const char* h = std::getenv("KTA_GEMM_L2HINT")) l2_hint = std::atoi(h) & 7;
}

// groups > 0 (expert GEMM, B [K, N] layout only): B is [groups, K, N] and rows
// [g * M / groups, (g + 1) * M / groups) of A and C use B[g]; M / groups must be a multiple
// of the 256-row pair tile.
template <bool BF16, bool B_KMAJOR, int PBN>
int launch_pair(const void* A, const void* B, void* C, int M, int N, int K, int64_t lda,
                int64_t ldb, int64_t ldc, cudaStream_t stream, int groups = 0) {
  using L = PairLayout<PBN>;
  const CUtensorMapDataType dt =
      BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb, tc;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(lda) * 2};
    const uint32_t box[2] = {BK, 128};
    int s = encode_tmap(&ta, dt, 2, A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  if (B_KMAJOR) {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldb) * 2};
    const uint32_t box[2] = {BK, PBN / 2};
    int s = encode_tmap(&tb, dt, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  } else if (groups > 0) {
    const uint64_t dims[3] = {static_cast<uint64_t>(N), static_cast<uint64_t>(K),
                              static_cast<uint64_t>(groups)};
    const uint64_t strides[2] = {static_cast<uint64_t>(ldb) * 2,
                                 static_cast<uint64_t>(ldb) * 2 * static_cast<uint64_t>(K)};
    const uint32_t box[3] = {64, BK, 1};
    int s = encode_tmap(&tb, dt, 3, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  } else {
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(K)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldb) * 2};
    const uint32_t box[2] = {64, BK};
    int s = encode_tmap(&tb, dt, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldc) * 2};
    const uint32_t box[2] = {EPI_COLS, 32};
    int s = encode_tmap(&tc, dt, 2, C, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  auto kernel = gemm_pair_kernel<BF16, B_KMAJOR, PBN>;
  int s = set_smem(kernel, L::ALLOC);
  if (s != KTA_OK) return s;
  const int tiles = ((M + P_BM - 1) / P_BM) * ((N + PBN - 1) / PBN);
  const int pairs = std::max(1, std::min(tiles, current_sm_count() / 2));
  int group_m = P_GROUP_M, l2_hint = 1;
  pair_raster_env(group_m, l2_hint);
  const int rows_per_group = groups > 0 ? M / groups : 0;
  return launch_ex(kernel, dim3(static_cast<unsigned>(2 * pairs)), dim3(NUM_THREADS), L::ALLOC,
                   stream, 2, ta, tb, tc, M, N, K, group_m, l2_hint, rows_per_group,
                   device_status_ptr());
}

// Estimated relative time of a tile width: waves x columns, discounted by the shared-memory
// traffic per tensor cycle (operand reads plus the TMA's writes: 128x256 tiles 192 B/clk,
// 128x128 256, 128x64 384). Measured: 128x128 tiles of a 4096^3 nn GEMM ran at 0.68 of the
// 128x256 rate.
inline double tile_cost(int M, int N, int BN, int sms) {
  const double eff = BN == 256 ? 1.0 : (BN == 128 ? 0.72 : 0.5);
  const long tiles = static_cast<long>((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const long waves = (tiles + sms - 1) / sms;
  return static_cast<double>(waves) * BN / eff;
}

// Selection of the 2-SM path: KTA_GEMM_PAIR=0 never; =force always (M >= 129; nn and expert
// GEMMs with 256-row multiples per expert included); unset: tn GEMMs whose 256x256 tiles
// fill the machine about as well as single-SM tiles.
inline int pair_mode() {
  const char* v = std::getenv("KTA_GEMM_PAIR");
  if (v == nullptr) return 1;
  if (v[0] == '0') return 0;
  if (v[0] == 'f') return 2;
  return 1;
}

// gemm_m16.cu: M <= 16 on mma.sync over every SM (KTA_ERR_UNSUPPORTED when N is too large)
template <bool BF16>
int launch_m16(const void* A, const void* B, void* C, int M, int N, int K, int64_t lda,
               int64_t ldb, int64_t ldc, cudaStream_t stream);

template <bool BF16, bool B_KMAJOR>
int dispatch(const void* A, const void* B, void* C, int64_t M64, int64_t N64, int64_t K64,
             int64_t lda, int64_t ldb, int64_t ldc, void* stream_v) {
  if (A == nullptr || B == nullptr || C == nullptr) return KTA_ERR_INVALID_ARG;
  if (M64 <= 0 || N64 <= 0 || K64 <= 0) return KTA_ERR_INVALID_ARG;
  if (M64 > (1 << 30) || N64 > (1 << 30) || K64 > (1 << 30)) return KTA_ERR_UNSUPPORTED;
  if (lda < K64 || ldc < N64 || (B_KMAJOR ? ldb < K64 : ldb < N64)) return KTA_ERR_INVALID_ARG;
  if (!aligned16(A) || !aligned16(B) || !aligned16(C)) return KTA_ERR_ALIGN;
  if (lda % 8 || ldb % 8 || ldc % 8) return KTA_ERR_ALIGN;
  int s = require_sm100();
  if (s != KTA_OK) return s;
  const int M = static_cast<int>(M64), N = static_cast<int>(N64), K = static_cast<int>(K64);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (B_KMAJOR && M <= 64) {
    if (M <= 16) {
      const int r = launch_m16<BF16>(A, B, C, M, N, K, lda, ldb, ldc, stream);
      if (r != KTA_ERR_UNSUPPORTED) return r;
      return launch_skinny<16, BF16>(A, B, C, M, N, K, lda, ldb, ldc, stream);
    }
    if (M <= 32) return launch_skinny<32, BF16>(A, B, C, M, N, K, lda, ldb, ldc, stream);
    if (M <= 48) return launch_skinny<48, BF16>(A, B, C, M, N, K, lda, ldb, ldc, stream);
    return launch_skinny<64, BF16>(A, B, C, M, N, K, lda, ldb, ldc, stream);
  }
  const int sms = std::max(1, current_sm_count());
  const int mode = pair_mode();
  if (mode == 2 && M > 128 && sms >= 2) {
    return launch_pair<BF16, B_KMAJOR, 256>(A, B, C, M, N, K, lda, ldb, ldc, stream);
  }
  // By default only tn takes pairs: with B an MN-major operand the pair kernel ran 8-10 %
  // below 128x256 single-SM tiles at 6144^3 and 8192^3 (it wins for tn: 1335 vs 1239)
  if (B_KMAJOR && mode == 1 && sms >= 2) {
    // 2-SM 256x256 tiles when they fill the machine about as well as 128x256 ones
    const long pair_tiles = static_cast<long>((M + 255) / 256) * ((N + 255) / 256);
    const long pair_waves = (pair_tiles + sms / 2 - 1) / (sms / 2);
    const long one_tiles = static_cast<long>((M + 127) / 128) * ((N + 255) / 256);
    const long one_waves = (one_tiles + sms - 1) / sms;
    if (pair_tiles >= sms / 2 && pair_waves <= one_waves) {
      return launch_pair<BF16, B_KMAJOR, 256>(A, B, C, M, N, K, lda, ldb, ldc, stream);
    }
  }
  const double c256 = tile_cost(M, N, 256, sms);
  const double c128 = tile_cost(M, N, 128, sms);
  const double c64 = tile_cost(M, N, 64, sms);
  if (c256 <= c128 && c256 <= c64) {
    return launch_main<256, 4, BF16, B_KMAJOR>(A, B, C, M, N, K, lda, ldb, ldc, stream);
  }
  if (c128 <= c64) {
    return launch_main<128, 6, BF16, B_KMAJOR>(A, B, C, M, N, K, lda, ldb, ldc, stream);
  }
  return launch_main<64, 8, BF16, B_KMAJOR>(A, B, C, M, N, K, lda, ldb, ldc, stream);
}

// MoE expert GEMM (KTA's moe_gemm, perfmodel/testset/gen.py:332-356): tokens grouped by
// expert, T / E rows each (a multiple of the 128-row tile, so no tile straddles two
// experts), C[rows of e] = A[rows of e] . W[e] with W [E, K, N]. One persistent launch over
// all experts' tiles; the producer picks W[e] per tile through a 3-D tensor map.
template <bool BF16>
int moe_dispatch(const void* A, const void* W, void* C, int64_t E64, int64_t T64, int64_t N64,
                 int64_t K64, void* stream_v) {
  if (A == nullptr || W == nullptr || C == nullptr) return KTA_ERR_INVALID_ARG;
  if (E64 <= 0 || T64 <= 0 || N64 <= 0 || K64 <= 0) return KTA_ERR_INVALID_ARG;
  if (E64 > 65536 || T64 > (1 << 30) || N64 > (1 << 30) || K64 > (1 << 30)) {
    return KTA_ERR_UNSUPPORTED;
  }
  if (T64 % E64 != 0 || (T64 / E64) % BM != 0) return KTA_ERR_UNSUPPORTED;
  if (!aligned16(A) || !aligned16(W) || !aligned16(C)) return KTA_ERR_ALIGN;
  if (K64 % 8 || N64 % 8) return KTA_ERR_ALIGN;
  int s = require_sm100();
  if (s != KTA_OK) return s;
  const int E = static_cast<int>(E64), T = static_cast<int>(T64), N = static_cast<int>(N64),
            K = static_cast<int>(K64);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  const int sms = std::max(1, current_sm_count());
  // 2-SM 256 x 128 tiles (both CTAs' rows in one expert) only with KTA_GEMM_PAIR=force: at
  // the test-set shape they ran at 530 TFLOP/s against 597 for single-SM tiles
  if (pair_mode() == 2 && (T / E) % P_BM == 0 && sms >= 2) {
    return launch_pair<BF16, false, 128>(A, W, C, T, N, K, K, N, N, stream, E);
  }
  if (tile_cost(T, N, 256, sms) <= tile_cost(T, N, 128, sms)) {
    return launch_main<256, 4, BF16, false>(A, W, C, T, N, K, K, N, N, stream, E);
  }
  return launch_main<128, 6, BF16, false>(A, W, C, T, N, K, K, N, N, stream, E);
}

}  // namespace gemm
}  // namespace kta

extern "C" int kta_moe_gemm_f16(const void* A, const void* W, void* C, int64_t E, int64_t T,
                                int64_t N, int64_t K, void* stream) {
  return kta::gemm::moe_dispatch<false>(A, W, C, E, T, N, K, stream);
}
extern "C" int kta_moe_gemm_bf16(const void* A, const void* W, void* C, int64_t E, int64_t T,
                                 int64_t N, int64_t K, void* stream) {
  return kta::gemm::moe_dispatch<true>(A, W, C, E, T, N, K, stream);
}
extern "C" void kta_so_moe_gemm_f16(uint64_t A, uint64_t W, uint64_t C, int32_t E, int32_t T,
                                    int32_t N, int32_t K) {
  kta::set_last_error(kta_moe_gemm_f16(reinterpret_cast<const void*>(A),
                                       reinterpret_cast<const void*>(W),
                                       reinterpret_cast<void*>(C), E, T, N, K, nullptr));
}

extern "C" {

int kta_gemm_bf16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                  int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  return kta::gemm::dispatch<true, true>(A, B, C, M, N, K, lda, ldb, ldc, stream);
}

int kta_gemm_f16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                 int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  return kta::gemm::dispatch<false, true>(A, B, C, M, N, K, lda, ldb, ldc, stream);
}

int kta_gemm_nn_bf16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                     int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  return kta::gemm::dispatch<true, false>(A, B, C, M, N, K, lda, ldb, ldc, stream);
}

int kta_gemm_nn_f16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                    int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  return kta::gemm::dispatch<false, false>(A, B, C, M, N, K, lda, ldb, ldc, stream);
}

// Reference `so` module entries (src/kta/measure/bench.py:94-98): device addresses and
// int32 shape scalars, dense row-major operands, default stream, no return value.
void kta_so_gemm_bf16(uint64_t A, uint64_t B, uint64_t C, int32_t M, int32_t N, int32_t K) {
  kta::set_last_error(kta_gemm_bf16(reinterpret_cast<const void*>(A),
                                    reinterpret_cast<const void*>(B),
                                    reinterpret_cast<void*>(C), M, N, K, K, K, N, nullptr));
}

void kta_so_gemm_f16(uint64_t A, uint64_t B, uint64_t C, int32_t M, int32_t N, int32_t K) {
  kta::set_last_error(kta_gemm_f16(reinterpret_cast<const void*>(A),
                                   reinterpret_cast<const void*>(B), reinterpret_cast<void*>(C),
                                   M, N, K, K, K, N, nullptr));
}

void kta_so_gemm_nn_f16(uint64_t A, uint64_t B, uint64_t C, int32_t M, int32_t N, int32_t K) {
  kta::set_last_error(kta_gemm_nn_f16(reinterpret_cast<const void*>(A),
                                      reinterpret_cast<const void*>(B),
                                      reinterpret_cast<void*>(C), M, N, K, K, N, N, nullptr));
}

void kta_so_gemm_nn_bf16(uint64_t A, uint64_t B, uint64_t C, int32_t M, int32_t N, int32_t K) {
  kta::set_last_error(kta_gemm_nn_bf16(reinterpret_cast<const void*>(A),
                                       reinterpret_cast<const void*>(B),
                                       reinterpret_cast<void*>(C), M, N, K, K, N, N, nullptr));
}

}  // extern "C"
