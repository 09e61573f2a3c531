// FP8 (e4m3) block-scaled GEMM on tcgen05, sm_100a.
//
//   C[M,N] (bf16) = sum_kb (A[:,kb] . B[:,kb]^T) * sa[m,kb] * sb[n/128,kb]
//
// A [M,K] and B [N,K] e4m3 (K-major); sa [M, ceil(K/128)] fp32 per 1x128 activation block,
// sb [ceil(N/128), ceil(K/128)] fp32 per 128x128 weight block. It replaces KTA's TileLang
// fp8gemm (perfmodel/testset/gen.py:306-329, C = A B^T, unscaled) with the block-scaled form.
// The scales are fp32 and not powers of two, so they cannot ride on the tensor core's own
// block-scale path; they are applied on the CUDA cores between 128-wide K blocks:
//
//   * persistent grid, grouped raster of 128 x 256 output tiles (two 128-wide weight-scale
//     blocks per tile); warp 0 TMA producer (128-byte swizzled K-major e4m3 tiles, one K
//     block = one 128-byte row per stage), warp 1 TMEM owner + single-thread
//     `tcgen05.mma.kind::f8f6f4` issuer;
//   * each K block's product goes to one of two TMEM partial buffers (2 x 256 columns), so
//     the tensor core works on block kb+1 while sixteen promotion warps fold block kb into
//     fp32 register accumulators: acc += partial * sa[m,kb] * sb[nb,kb] with packed f32x2
//     FMAs (each thread one row, 64 columns inside one weight block; four warps per SMSP
//     keep the TMEM loads of one warp behind the FMAs of the others);
//   * the tile's accumulators go straight to global memory as bf16 rows;
//   * every mbarrier wait is bounded.
#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "kta_common.cuh"
#include "kta_host.h"

namespace kta {
namespace fp8 {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;               // e4m3 elements per stage = one scale block = 128 bytes
constexpr int UMMA_K = 32;            // K per tcgen05.mma of kind::f8f6f4
constexpr int STAGES = 4;
constexpr int PROMO_WARPS = 16;      // four per SMSP: TMEM load latency hides behind FMAs
constexpr int PROMO_COLS = 4 * BN / PROMO_WARPS;  // 64 columns of one row per thread
constexpr int NUM_THREADS = 64 + PROMO_WARPS * 32;
constexpr int GROUP_M = 16;

enum : unsigned int {
  SITE_PROD = 0x501,
  SITE_MMA_FULL = 0x502,
  SITE_MMA_TEMPTY = 0x503,
  SITE_PROMO = 0x504,
};

struct Layout {
  static constexpr int A_BYTES = BM * BK;        // 16 KB
  static constexpr int B_BYTES = BN * BK;        // 32 KB
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_BAR = OFF_B + STAGES * B_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 4;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int TOTAL = OFF_MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;
  static_assert(ALLOC <= 232448, "shared memory budget of one sm_100 CTA");
};

struct Params {
  const float* sa;     // [M, KB]
  const float* sb;     // [NB, KB]
  __nv_bfloat16* c;    // [M, N]
  int M, N, K, KB, NB;
  int items;           // work items of this launch (tiles, or quarters of tiles)
  int tile_base;       // the quarter launch: raster index of the first tile it cuts up
  int prefetch;        // A and B exceed kPrefetchMinBytes: L2 prefetch before the wait
  unsigned int* status;
};

// The quarter launch: tiles that would fill only part of the last round of the main launch
// are cut into 128 x 64 quarters and run by a second launch on the SMs the main one has left
// idle, so that the round takes about a quarter of the time.
constexpr int SUB = 4;
constexpr int SUB_N = BN / SUB;

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& mb,
                                            int& nb) {
  const int per_group = GROUP_M * tiles_n;
  const int group = tile / per_group;
  const int first_m = group * GROUP_M;
  const int gsz = min(tiles_m - first_m, GROUP_M);
  const int r = tile - group * per_group;
  mb = first_m + r % gsz;
  nb = r / gsz;
}

// QTR: items are 128 x 64 quarters of the tiles from p.tile_base on (B through a map with a
// 64-row box; each promotion warp holds 16 of the quarter's columns); otherwise whole tiles.
template <bool QTR>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Layout::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Layout::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Layout::OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], PROMO_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);  // two partial buffers of 256 columns
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int tiles_m = (p.M + BM - 1) / BM;
  const int tiles_n = (p.N + BN - 1) / BN;
  const int num_tiles = p.items;
  const int KB = p.KB;
  // tile (mb, nb) of item `it`, and the first accumulator / output column of the item
  auto coords = [&](int it, int& mb, int& nb, int& col) {
    if constexpr (QTR) {
      tile_coords(p.tile_base + it / SUB, tiles_m, tiles_n, mb, nb);
      col = (it % SUB) * SUB_N;
    } else {
      tile_coords(it, tiles_m, tiles_n, mb, nb);
      col = 0;
    }
  };
  pdl_launch_dependents();
  if (p.prefetch && warp == 0 && lane == 0 && static_cast<int>(blockIdx.x) < num_tiles) {
    // While the previous grid finishes, pull the first ring's K blocks of this CTA's first
    // item into L2 (a prefetch writes nothing, so it may precede the wait).
    int mb, nb, col;
    coords(blockIdx.x, mb, nb, col);
    for (int kb = 0; kb < KB && kb < STAGES; ++kb) {
      tma_prefetch_l2_2d(&tmA, kb * BK, mb * BM);
      tma_prefetch_l2_2d(&tmB, kb * BK, nb * BN + col);
    }
  }
  pdl_wait();  // the previous grid's writes (this launch's inputs) are visible from here on

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      constexpr int b_bytes = QTR ? Layout::B_BYTES / SUB : Layout::B_BYTES;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mb, nb, col;
        coords(tile, mb, nb, col);
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status, SITE_PROD)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Layout::A_BYTES + b_bytes);
          tma_load_2d(&tmA, &full[stage], smem + Layout::OFF_A + stage * Layout::A_BYTES,
                      kb * BK, mb * BM);
          tma_load_2d(&tmB, &full[stage], smem + Layout::OFF_B + stage * Layout::B_BYTES,
                      kb * BK, nb * BN + col);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // e4m3 x e4m3 -> f32
      constexpr uint32_t idesc = make_idesc(BM, QTR ? SUB_N : BN, 0u, 0u, 0u, 0u);
      int stage = 0;
      uint32_t phase = 0;
      int buf = 0;
      uint32_t bphase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&tempty[buf], bphase ^ 1u, abort_flag, p.status, SITE_MMA_TEMPTY) ||
              !mbar_wait(&full[stage], phase, abort_flag, p.status, SITE_MMA_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + Layout::OFF_A + stage * Layout::A_BYTES);
          const uint32_t b0 = smem_u32(smem + Layout::OFF_B + stage * Layout::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            umma_f8(tmem + buf * BN, sdesc_sw128(a0 + k * UMMA_K, 16, 1024),
                    sdesc_sw128(b0 + k * UMMA_K, 16, 1024), idesc, k > 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          umma_commit(&tfull[buf]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          buf ^= 1;
          if (buf == 0) bphase ^= 1u;
        }
      }
    }
  } else {
    // ---------------- promotion + epilogue: thread = output row, 64 columns ----------------
    const int quarter = warp & 3;
    const int cg = (warp - 2) >> 2;    // 64-column group of the tile (0..3)
    const int half = cg >> 1;          // which 128-column weight block of the tile
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    int buf = 0;
    uint32_t bphase = 0;
    bool ok = true;
    // columns of the accumulator this warp promotes (a quarter: 16 of its 64)
    constexpr int COLS = QTR ? SUB_N / 4 : PROMO_COLS;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      int mb, nb, col;
      coords(tile, mb, nb, col);
      const int m = mb * BM + row;
      const int c0 = QTR ? cg * COLS : cg * PROMO_COLS;  // first accumulator column
      const int nblk = QTR ? (nb * BN + col) / 128 : nb * 2 + half;  // weight-scale block
      const bool row_in = m < p.M;
      const bool blk_in = nblk < p.NB;
      // 32-bit offsets into the scale arrays (the launch checks M x KB and NB x KB < 2^31);
      // the bases stay kernel parameters. The scales of K block kb+2 are loaded while block
      // kb is folded and multiplied only when used, so no load latency lands on the
      // promotion path.
      const bool live = row_in && blk_in;
      const int sa_off = live ? m * KB : 0;
      const int sb_off = live ? nblk * KB : 0;
      uint64_t acc[COLS / 2];  // packed pairs of fp32 accumulators
#pragma unroll
      for (int i = 0; i < COLS / 2; ++i) acc[i] = 0ull;
      float a0 = 0.f, b0 = 0.f, a1 = 0.f, b1 = 0.f;  // scales of blocks kb and kb+1
      if (live) {
        a0 = __ldg(p.sa + sa_off);
        b0 = __ldg(p.sb + sb_off);
        if (KB > 1) {
          a1 = __ldg(p.sa + sa_off + 1);
          b1 = __ldg(p.sb + sb_off + 1);
        }
      }
      for (int kb = 0; kb < KB; ++kb) {
        const float scale = a0 * b0;
        a0 = a1;
        b0 = b1;
        if (live && kb + 2 < KB) {
          a1 = __ldg(p.sa + sa_off + kb + 2);
          b1 = __ldg(p.sb + sb_off + kb + 2);
        }
        if (!mbar_wait(&tfull[buf], bphase, abort_flag, p.status, SITE_PROMO)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t t = tmem + lane_base + buf * BN + c0;
        const uint64_t s2 = f2(scale, scale);
#pragma unroll
        for (int c = 0; c < COLS; c += 16) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(t + c, r);
          tmem_ld_wait();
          reg_fence(r);
          if (c + 16 == COLS) {
            // the buffer's last columns are in registers: hand it back before the last FMAs
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            acc[c / 2 + i] = fma2(f2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), s2,
                                  acc[c / 2 + i]);
          }
        }
        buf ^= 1;
        if (buf == 0) bphase ^= 1u;
      }
      if (!ok) break;
      const int n0 = nb * BN + col + c0;
      if (row_in && n0 < p.N) {
        __nv_bfloat16* crow = p.c + static_cast<long long>(m) * p.N + n0;
        uint32_t pk[COLS / 2];
#pragma unroll
        for (int i = 0; i < COLS / 2; ++i) {
          float x0, x1;
          f2_split(acc[i], x0, x1);
          pk[i] = pack_bf16x2(x0, x1);
        }
#pragma unroll
        for (int c = 0; c < COLS; c += 8) {
          if (n0 + c < p.N) {
            *reinterpret_cast<uint4*>(crow + c) =
                make_uint4(pk[c / 2], pk[c / 2 + 1], pk[c / 2 + 2], pk[c / 2 + 3]);
          }
        }
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

int launch(const void* A, const void* sa, const void* B, const void* sb, void* C, int64_t M64,
           int64_t N64, int64_t K64, cudaStream_t stream) {
  if (!A || !sa || !B || !sb || !C) return KTA_ERR_INVALID_ARG;
  if (M64 <= 0 || N64 <= 0 || K64 <= 0) return KTA_ERR_INVALID_ARG;
  if (M64 > (1 << 30) || N64 > (1 << 30) || K64 > (1 << 30)) return KTA_ERR_UNSUPPORTED;
  // scale arrays indexed with 32-bit offsets (an A or B this large would exceed 256 GB)
  if (M64 * ((K64 + BK - 1) / BK) >= (int64_t{1} << 31) ||
      ((N64 + 127) / 128) * ((K64 + BK - 1) / BK) >= (int64_t{1} << 31)) {
    return KTA_ERR_UNSUPPORTED;
  }
  if (K64 % 16 != 0 || N64 % 8 != 0) return KTA_ERR_ALIGN;
  if (!aligned16(A) || !aligned16(B) || !aligned16(C) ||
      (reinterpret_cast<uintptr_t>(sa) & 3) || (reinterpret_cast<uintptr_t>(sb) & 3)) {
    return KTA_ERR_ALIGN;
  }
  int s = require_sm100();
  if (s != KTA_OK) return s;
  const int M = static_cast<int>(M64), N = static_cast<int>(N64), K = static_cast<int>(K64);
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K)};
    const uint32_t box[2] = {BK, BM};
    s = encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, A, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  CUtensorMap tbq;  // B with a 64-row box, for the quarter launch
  for (int i = 0; i < 2; ++i) {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K)};
    const uint32_t box[2] = {BK, static_cast<uint32_t>(i == 0 ? BN : SUB_N)};
    s = encode_tmap(i == 0 ? &tb : &tbq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, B, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  Params prm;
  prm.sa = static_cast<const float*>(sa);
  prm.sb = static_cast<const float*>(sb);
  prm.c = static_cast<__nv_bfloat16*>(C);
  prm.M = M;
  prm.N = N;
  prm.K = K;
  prm.KB = (K + BK - 1) / BK;
  prm.NB = (N + 127) / 128;
  prm.prefetch = (M64 + N64) * K64 > kPrefetchMinBytes ? 1 : 0;
  prm.status = device_status_ptr();
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int sms = std::max(1, current_sm_count());
  // The tiles of a ragged last round (4096 x 7168: 896 tiles = 6 rounds of 148 + 8) go to a
  // second launch as quarters when those fit in one round on the SMs (8 -> 32 quarters);
  // KTA_FP8_SPLIT=0 keeps them whole (comparison runs).
  const int rem = tiles > sms ? tiles % sms : 0;
  const char* split = std::getenv("KTA_FP8_SPLIT");
  const bool quarters = rem > 0 && rem * SUB <= sms && (split == nullptr || split[0] != '0');
  const int main_tiles = quarters ? tiles - rem : tiles;
  s = set_kernel_smem(reinterpret_cast<const void*>(fp8_gemm_kernel<false>), Layout::ALLOC);
  if (s != KTA_OK) return s;
  prm.items = main_tiles;
  prm.tile_base = 0;
  s = launch_ex(fp8_gemm_kernel<false>, dim3(std::min(main_tiles, sms)), dim3(NUM_THREADS),
                Layout::ALLOC, stream, 1, ta, tb, prm);
  if (s != KTA_OK || !quarters) return s;
  s = set_kernel_smem(reinterpret_cast<const void*>(fp8_gemm_kernel<true>), Layout::ALLOC);
  if (s != KTA_OK) return s;
  prm.items = rem * SUB;
  prm.tile_base = main_tiles;
  return launch_ex(fp8_gemm_kernel<true>, dim3(rem * SUB), dim3(NUM_THREADS), Layout::ALLOC,
                   stream, 1, ta, tbq, prm);
}

}  // namespace fp8
}  // namespace kta

extern "C" int kta_gemm_fp8_blockscaled(const void* A, const void* sa, const void* B,
                                        const void* sb, void* C, int64_t M, int64_t N, int64_t K,
                                        void* stream) {
  return kta::fp8::launch(A, sa, B, sb, C, M, N, K, static_cast<cudaStream_t>(stream));
}
