// GEMM with a 4-bit B dequantised in the main loop, sm_100a:
//
//   C[M,N] (f16) = A[M,K] (f16) . B^T,   B[n,k] = decode(Bq[n, k/2] nibble k%2) * Sc[n, k/G]
//
//   INT4 (w4a16): decode(x) = x - 8, G = group (KTA's w4gemm, perfmodel/testset/gen.py:359-414)
//   E2M1 (NVFP4): decode(x) = e2m1 value of x, G = 16 (KTA's nvfp4gemm, gen.py:744-778)
//
// Two 4-bit elements per byte, the lower nibble first; the scale is f16 and the product is
// rounded once to f16, as the reference computes it. The tensor cores take f16 x f16
// (tcgen05.mma kind::f16, fp32 accumulator in TMEM), so B is expanded in shared memory:
//
//   * warp 0: TMA producer; per 64-deep K stage the A tile (128 x 64 f16, 128-byte swizzle)
//     and the packed B tile (128 rows x 32 bytes), 6-stage ring;
//   * warps 6-13: converters; each thread expands 32 elements of one B row (16 bytes in,
//     four 16-byte swizzled chunks out) into the stage's f16 B tile, K-major with the 128-byte
//     swizzle the MMA descriptor expects, then a proxy fence and one arrival per warp;
//   * warp 1: TMEM owner and single-thread MMA issuer (4 MMAs of K = 16 per stage) into two
//     accumulators of 128 columns; warps 2-5: epilogue (TMEM -> f16 -> global rows);
//   * persistent grid, grouped raster of 128 x 128 tiles; every mbarrier wait is bounded.
//
// Algorithmic work per launch: 2 M N K FLOP; bytes 2 M K + N K / 2 + 2 N K / G + 2 M N.
#include <algorithm>

#include "kta_common.cuh"
#include "kta_host.h"

namespace kta {
namespace dq {

constexpr int BM = 128, BN = 128, BK = 64;
constexpr int STAGES = 6;
constexpr int CONV_WARPS = 8;
constexpr int EPI_WARPS = 4;
constexpr int NUM_THREADS = 32 * (2 + EPI_WARPS + CONV_WARPS);  // 448
constexpr int CONV_FIRST_WARP = 2 + EPI_WARPS;
constexpr int GROUP_M = 16;

enum : unsigned int {
  SITE_PROD = 0x701,
  SITE_CONV = 0x702,
  SITE_MMA_FULL = 0x703,
  SITE_MMA_CONV = 0x704,
  SITE_MMA_TEMPTY = 0x705,
  SITE_EPI = 0x706,
};

struct Layout {
  static constexpr int A_BYTES = BM * BK * 2;   // 16 KB, swizzled
  static constexpr int Q_BYTES = BN * BK / 2;   // 4 KB packed B
  static constexpr int B_BYTES = BN * BK * 2;   // 16 KB expanded B, swizzled
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_Q = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_BAR = OFF_Q + STAGES * Q_BYTES;
  // full[S], conv[S], empty[S], tfull[2], tempty[2]
  static constexpr int NUM_BARS = 3 * STAGES + 4;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int TOTAL = OFF_MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;
  static_assert(ALLOC <= 232448, "shared memory budget of one sm_100 CTA");
};

struct Params {
  const __half* sc;   // [N, K / G]
  __half* c;          // [M, N]
  int M, N, K, group;
  unsigned int* status;
};

__device__ __forceinline__ void tile_of(int tile, int tiles_m, int tiles_n, int& mb, int& nb) {
  const int per_group = GROUP_M * tiles_n;
  const int g = tile / per_group;
  const int first_m = g * GROUP_M;
  const int gsz = min(tiles_m - first_m, GROUP_M);
  const int r = tile - g * per_group;
  mb = first_m + r % gsz;
  nb = r / gsz;
}

__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t bits) {
  return (a & mask) | bits;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Eight int4 elements (one 32-bit word: k0 in bits 0-3 ... k7 in bits 28-31) times the f16
// scale pair s2 -> four f16x2 words (k0,k1), (k2,k3), (k4,k5), (k6,k7). 0x6400 | x is the f16
// 1024 + x (x < 16, exact: the spacing of f16 in [1024, 2048) is 1), so subtracting 1032 gives
// x - 8 exactly; the one rounding is the product with s, for every scale (subnormal included).
__device__ __forceinline__ void int4x8_to_f16(uint32_t w, uint32_t s2, uint32_t (&o)[4]) {
  const uint32_t x04 = lop_and_or(w, 0x000F000Fu, 0x64006400u);          // (k0, k4) + 1024
  const uint32_t x15 = lop_and_or(w >> 4, 0x000F000Fu, 0x64006400u);     // (k1, k5) + 1024
  const uint32_t x26 = lop_and_or(w >> 8, 0x000F000Fu, 0x64006400u);     // (k2, k6) + 1024
  const uint32_t x37 = lop_and_or(w >> 12, 0x000F000Fu, 0x64006400u);    // (k3, k7) + 1024
  const uint32_t v04 = hmul2(hsub2(x04, 0x64086408u), s2);
  const uint32_t v15 = hmul2(hsub2(x15, 0x64086408u), s2);
  const uint32_t v26 = hmul2(hsub2(x26, 0x64086408u), s2);
  const uint32_t v37 = hmul2(hsub2(x37, 0x64086408u), s2);
  o[0] = prmt(v04, v15, 0x5410u);  // (k0, k1)
  o[1] = prmt(v26, v37, 0x5410u);  // (k2, k3)
  o[2] = prmt(v04, v15, 0x7632u);  // (k4, k5)
  o[3] = prmt(v26, v37, 0x7632u);  // (k6, k7)
}

// Eight e2m1 elements (one 32-bit word, lower nibble first) times s2 -> four f16x2 words.
__device__ __forceinline__ void e2m1x8_to_f16(uint32_t w, uint32_t s2, uint32_t (&o)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t h;
    asm("{\n"
        " .reg .b8 b;\n"
        " cvt.u8.u32 b, %1;\n"
        " cvt.rn.f16x2.e2m1x2 %0, b;\n"
        "}\n"
        : "=r"(h)
        : "r"(w >> (8 * i)));
    o[i] = hmul2(h, s2);
  }
}

__device__ __forceinline__ uint32_t half2_bits(__half a) {
  const uint16_t u = __half_as_ushort(a);
  return static_cast<uint32_t>(u) | (static_cast<uint32_t>(u) << 16);
}

template <bool E2M1>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    dq_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmQ,
                   const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Layout::OFF_BAR);
  uint64_t* conv = full + STAGES;
  uint64_t* empty = conv + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Layout::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Layout::OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], CONV_WARPS);
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
    tma_prefetch_desc(&tmQ);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int tiles_m = (p.M + BM - 1) / BM;
  const int tiles_n = (p.N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = p.K / BK;

  if (warp == 0) {
    // ---------------- TMA producer: A and packed B ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_of(tile, tiles_m, tiles_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status, SITE_PROD)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Layout::A_BYTES + Layout::Q_BYTES);
          tma_load_2d(&tmA, &full[stage], smem + Layout::OFF_A + stage * Layout::A_BYTES,
                      kb * BK, mb * BM);
          tma_load_2d(&tmQ, &full[stage], smem + Layout::OFF_Q + stage * Layout::Q_BYTES,
                      kb * (BK / 2), nb * BN);
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
      constexpr uint32_t idesc = make_idesc(BM, BN, 0u, 0u, 0u, 0u);  // f16 x f16, K-major
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.status, SITE_MMA_TEMPTY)) {
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status, SITE_MMA_FULL) ||
              !mbar_wait(&conv[stage], phase, abort_flag, p.status, SITE_MMA_CONV)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + Layout::OFF_A + stage * Layout::A_BYTES);
          const uint32_t b0 = smem_u32(smem + Layout::OFF_B + stage * Layout::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma_f16(d, sdesc_sw128(a0 + k * 32, 16, 1024), sdesc_sw128(b0 + k * 32, 16, 1024),
                     idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else if (warp < CONV_FIRST_WARP) {
    // ---------------- epilogue: thread = output row ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mb, nb;
      tile_of(tile, tiles_m, tiles_n, mb, nb);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status, SITE_EPI)) break;
      tc_fence_after();
      const int m = mb * BM + row;
      const uint32_t t = tmem + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t + c, r);
        tmem_ld_wait();
        reg_fence(r);
        const int n0 = nb * BN + c;
        if (m < p.M && n0 < p.N) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const __half2 h = __floats2half2_rn(__uint_as_float(r[2 * i]),
                                                __uint_as_float(r[2 * i + 1]));
            pk[i] = *reinterpret_cast<const uint32_t*>(&h);
          }
          __half* crow = p.c + static_cast<long long>(m) * p.N + n0;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (n0 + 8 * i < p.N) {
              *reinterpret_cast<uint4*>(crow + 8 * i) =
                  make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  } else {
    // ---------------- converters: thread = half of one B row of the stage ----------------
    const int ct = threadIdx.x - CONV_FIRST_WARP * 32;   // 0 .. 255
    const int n_local = ct >> 1;                         // B row within the tile
    const int half = ct & 1;                             // k 0-31 or 32-63 of the stage
    const int kgroups = p.K / p.group;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      int mb, nb;
      tile_of(tile, tiles_m, tiles_n, mb, nb);
      const int n = nb * BN + n_local;
      const __half* sc_row = p.sc + static_cast<long long>(min(n, p.N - 1)) * kgroups;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int k0 = kb * BK + half * 32;              // first k of this thread's 32
        // scales of the 32 elements: one when G >= 32, two (k0 and k0 + 16) when G = 16
        const __half s_a = __ldg(sc_row + k0 / p.group);
        const __half s_b = __ldg(sc_row + (k0 + 16) / p.group);
        if (!mbar_wait(&full[stage], phase, abort_flag, p.status, SITE_CONV)) {
          ok = false;
          break;
        }
        const uint4 in = *reinterpret_cast<const uint4*>(
            smem + Layout::OFF_Q + stage * Layout::Q_BYTES + n_local * (BK / 2) + half * 16);
        const uint32_t w[4] = {in.x, in.y, in.z, in.w};  // 8 elements each, k order
        const uint32_t b_row = smem_u32(smem + Layout::OFF_B + stage * Layout::B_BYTES) +
                               static_cast<uint32_t>(n_local) * 128u;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t s2 = half2_bits(i < 2 ? s_a : s_b);
          uint32_t o[4];
          if constexpr (E2M1) {
            e2m1x8_to_f16(w[i], s2, o);
          } else {
            int4x8_to_f16(w[i], s2, o);
          }
          // 16-byte chunk (half * 4 + i) of the row, 128-byte swizzle: chunk ^ (row & 7)
          const uint32_t chunk = static_cast<uint32_t>(half * 4 + i) ^ static_cast<uint32_t>(n_local & 7);
          st_shared_v4(b_row + (chunk << 4), o[0], o[1], o[2], o[3]);
        }
        fence_proxy_async_smem();  // generic-proxy writes -> the tensor core's reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

template <bool E2M1>
int launch(const void* A, const void* Bq, const void* Sc, void* C, int64_t M64, int64_t N64,
           int64_t K64, int64_t group, void* stream_v) {
  if (!A || !Bq || !Sc || !C) return KTA_ERR_INVALID_ARG;
  if (M64 <= 0 || N64 <= 0 || K64 <= 0) return KTA_ERR_INVALID_ARG;
  if (group < 16 || group > 4096 || (group & (group - 1)) != 0) return KTA_ERR_INVALID_ARG;
  if (M64 > (1 << 30) || N64 > (1 << 30) || K64 > (1 << 30)) return KTA_ERR_UNSUPPORTED;
  if (K64 % BK != 0 || K64 % group != 0) return KTA_ERR_ALIGN;  // whole stages and groups
  if (N64 % 8 != 0) return KTA_ERR_ALIGN;
  if (!aligned16(A) || !aligned16(Bq) || !aligned16(C) ||
      (reinterpret_cast<uintptr_t>(Sc) & 1)) {
    return KTA_ERR_ALIGN;
  }
  int s = require_sm100();
  if (s != KTA_OK) return s;
  const int M = static_cast<int>(M64), N = static_cast<int>(N64), K = static_cast<int>(K64);
  CUtensorMap ta, tq;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {BK, BM};
    s = encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K / 2), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K / 2)};
    const uint32_t box[2] = {BK / 2, BN};
    s = encode_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, Bq, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_NONE);
    if (s != KTA_OK) return s;
  }
  Params prm;
  prm.sc = static_cast<const __half*>(Sc);
  prm.c = static_cast<__half*>(C);
  prm.M = M;
  prm.N = N;
  prm.K = K;
  prm.group = static_cast<int>(group);
  prm.status = device_status_ptr();
  auto kernel = dq_gemm_kernel<E2M1>;
  s = set_kernel_smem(reinterpret_cast<const void*>(kernel), Layout::ALLOC);
  if (s != KTA_OK) return s;
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = std::max(1, std::min(tiles, current_sm_count()));
  kernel<<<grid, NUM_THREADS, Layout::ALLOC, static_cast<cudaStream_t>(stream_v)>>>(ta, tq, prm);
  return launch_status();
}

}  // namespace dq
}  // namespace kta

extern "C" int kta_gemm_w4a16_f16(const void* A, const void* Bq, const void* Sc, void* C,
                                  int64_t M, int64_t N, int64_t K, int64_t group, void* stream) {
  return kta::dq::launch<false>(A, Bq, Sc, C, M, N, K, group, stream);
}
extern "C" int kta_gemm_nvfp4_f16(const void* A, const void* Bq, const void* Sc, void* C,
                                  int64_t M, int64_t N, int64_t K, void* stream) {
  return kta::dq::launch<true>(A, Bq, Sc, C, M, N, K, 16, stream);
}
extern "C" void kta_so_w4gemm_f16(uint64_t A, uint64_t Bq, uint64_t Sc, uint64_t C, int32_t M,
                                  int32_t N, int32_t K) {
  kta::set_last_error(kta_gemm_w4a16_f16(reinterpret_cast<const void*>(A),
                                         reinterpret_cast<const void*>(Bq),
                                         reinterpret_cast<const void*>(Sc),
                                         reinterpret_cast<void*>(C), M, N, K, 32, nullptr));
}
extern "C" void kta_so_nvfp4gemm_f16(uint64_t A, uint64_t Bq, uint64_t Sc, uint64_t C, int32_t M,
                                     int32_t N, int32_t K) {
  kta::set_last_error(kta_gemm_nvfp4_f16(reinterpret_cast<const void*>(A),
                                         reinterpret_cast<const void*>(Bq),
                                         reinterpret_cast<const void*>(Sc),
                                         reinterpret_cast<void*>(C), M, N, K, nullptr));
}
