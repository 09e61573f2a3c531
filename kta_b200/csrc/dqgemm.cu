// GEMM with a 4-bit B dequantised in the main loop, sm_100a:
//
//   C[M,N] (f16) = A[M,K] (f16) . B^T,   B[n,k] = decode(Bq[n, k/2] nibble k%2) * Sc[n, k/G]
//
//   INT4 (w4a16): decode(x) = x - 8, G = group (KTA's w4gemm, perfmodel/testset/gen.py:359-414)
//   E2M1 (NVFP4): decode(x) = e2m1 value of x, G = 16 (KTA's nvfp4gemm, gen.py:744-778)
//
// Two 4-bit elements per byte, the lower nibble first; the scale is f16 and the product is
// rounded once to f16, as the reference computes it. The tensor cores take f16 x f16
// (tcgen05.mma kind::f16, fp32 accumulator in TMEM) with the expanded B as the MMA's A
// operand read from TMEM, so the product is formed transposed, D[n, m] = B[n, :] . A[m, :]:
//
//   * warp 0: TMA producer; per 64-deep K stage the A tile (up to 256 rows x 64 f16, 128-byte
//     swizzle; the MMA's B operand) and the packed B tile (128 rows x 32 bytes), 6 stages;
//   * warp 1: TMEM owner and single-thread MMA issuer, M = 128 (B rows) x N = the m tile
//     (256, or M rounded up to 16 when one tile covers M), 4 MMAs of K = 16 per stage;
//   * warps 2-17: workers in four stage groups (one warp per TMEM lane quarter per group):
//     the stages are dealt round-robin to the groups, a thread expands all 64 codes of its B
//     row with scales fetched one group-turn ahead and stores them with tcgen05.st into the
//     stage's TMEM slot; at the end of a tile all sixteen drain the accumulator (64 columns
//     each; neighbouring lanes swap halves so each stores an (n, n + 1) pair of C[m, :]);
//   * persistent grid, grouped raster of tiles; every mbarrier wait is bounded.
//
// Shared memory carries only the TMA writes and the tensor core's reads of A (68 KB per stage
// of 128 x 256 x 64): the expanded B goes from registers to TMEM. Writing it to shared memory
// instead (and reading it back as an MMA operand) makes shared-memory bandwidth the bound.
//
// Algorithmic work per launch: 2 M N K FLOP; bytes 2 M K + N K / 2 + 2 N K / G + 2 M N.
#include <algorithm>

#include "kta_common.cuh"
#include "kta_host.h"

namespace kta {
namespace dq {

constexpr int BN = 128;      // rows of B per tile: the MMA's M, TMEM lanes
constexpr int MT_MAX = 256;  // rows of A per tile: the MMA's N, TMEM columns of D
constexpr int BK = 64;
constexpr int STAGES = 6;
constexpr int WORK_GROUPS = 4;                       // stages being expanded at once
constexpr int WORK_WARPS = 4 * WORK_GROUPS;           // one warp per TMEM lane quarter per group
constexpr int NUM_THREADS = 32 * (2 + WORK_WARPS);    // 576
constexpr int GROUP_M = 16;
// TMEM: D in columns [0, 256), the expanded B of stage s in [256 + 32 s, 256 + 32 (s + 1))
// (128 rows x 64 f16, two per 32-bit column)
constexpr int TMEM_B_COL = MT_MAX;
constexpr int TMEM_COLS = 512;
static_assert(TMEM_B_COL + STAGES * (BK / 2) <= TMEM_COLS, "TMEM budget of one SM");
static_assert(MT_MAX / WORK_GROUPS == 64, "each worker warp drains two 32-column loads");

enum : unsigned int {
  SITE_PROD = 0x701,
  SITE_CONV = 0x702,
  SITE_MMA_FULL = 0x703,
  SITE_MMA_CONV = 0x704,
  SITE_MMA_TEMPTY = 0x705,
  SITE_EPI = 0x706,
};

struct Layout {
  static constexpr int A_BYTES = MT_MAX * BK * 2;  // 32 KB of A rows, swizzled
  static constexpr int Q_BYTES = BN * BK / 2;      // 4 KB of packed B
  static constexpr int OFF_A = 0;
  static constexpr int OFF_Q = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_BAR = OFF_Q + STAGES * Q_BYTES;
  // full[S], conv[S], empty[S], tfull, tempty
  static constexpr int NUM_BARS = 3 * STAGES + 2;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int TOTAL = OFF_MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;
  static_assert(ALLOC <= 232448, "shared memory budget of one sm_100 CTA");
};

struct Params {
  const __half* sc;   // [N, K / G]
  __half* c;          // [M, N]
  int M, N, K, group;
  int m_tile;         // rows of A per tile (the MMA's N)
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

// One CTA per SM; tile = 128 rows of B (n) x up to 256 rows of A (m), transposed product:
//   D[n, m] (TMEM, fp32) += Bdq[n, k] (TMEM, f16) . A[m, k] (shared memory, f16)
// so the expanded B never touches shared memory: the converters store it into TMEM with
// tcgen05.st and the MMA reads it from there (A operand from TMEM), while TMA brings the
// activation tile as the MMA's B operand. A 64-deep stage moves 32 KB of A and 4 KB of codes
// into shared memory and 32 KB of A out to the tensor core for 128 x 256 x 64 of work.
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
  uint64_t* tempty = tfull + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Layout::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Layout::OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);  // the four warps of the stage's group
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, WORK_WARPS);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmQ);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_launch_dependents();
  pdl_wait();  // the previous grid's writes (this launch's inputs) are visible from here on
  const int mt = p.m_tile;
  const int tiles_m = (p.M + mt - 1) / mt;
  const int tiles_n = (p.N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = p.K / BK;

  if (warp == 0) {
    // ---------------- TMA producer: A rows (the MMA's B operand) and packed B rows ----------
    if (lane == 0) {
      const uint32_t bytes = static_cast<uint32_t>(mt) * BK * 2 + Layout::Q_BYTES;
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
          mbar_arrive_expect_tx(&full[stage], bytes);
          tma_load_2d(&tmA, &full[stage], smem + Layout::OFF_A + stage * Layout::A_BYTES,
                      kb * BK, mb * mt);
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
    // ---------------- MMA issuer: M = 128 (B rows, TMEM), N = m tile (A rows, smem) ---------
    if (lane == 0) {
      const uint32_t idesc = make_idesc(BN, mt, 0u, 0u, 0u, 0u);  // f16 x f16, K-major
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(tempty, acc_phase ^ 1u, abort_flag, p.status, SITE_MMA_TEMPTY)) break;
        tc_fence_after();
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status, SITE_MMA_FULL) ||
              !mbar_wait(&conv[stage], phase, abort_flag, p.status, SITE_MMA_CONV)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b0 = smem_u32(smem + Layout::OFF_A + stage * Layout::A_BYTES);
          const uint32_t a0 = tmem + static_cast<uint32_t>(TMEM_B_COL + stage * (BK / 2));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma_f16_tmem_a(tmem, a0 + k * 8, sdesc_sw128(b0 + k * 32, 16, 1024), idesc,
                            (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);  // frees the stage's shared memory and TMEM slot
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(tfull);
        acc_phase ^= 1u;
      }
    }
  } else {
    // ---------------- workers: expand B into TMEM, then drain D at the end of each tile ------
    // Warp w serves TMEM lane quarter q = w % 4 (the lanes a warp may access) and stage group
    // g: the CTA's stage sequence is dealt round-robin to the WORK_GROUPS groups, so that many
    // stages are being expanded at once; a thread expands all 64 codes of its B row n.
    const int q = warp & 3;
    const int g = (warp - 2) >> 2;
    const int n_local = q * 32 + lane;
    const bool odd = lane & 1;
    const int kgroups = p.K / p.group;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q * 32) << 16);
    long long it_base = 0;  // index of the tile's first stage in the CTA's stage sequence
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      int mb, nb;
      tile_of(tile, tiles_m, tiles_n, mb, nb);
      const unsigned short* sc_row = reinterpret_cast<const unsigned short*>(p.sc) +
                                     static_cast<long long>(min(nb * BN + n_local, p.N - 1)) * kgroups;
      // this group's first stage of the tile, and the scales of the four 16-code groups
      int kb = static_cast<int>(((g - it_base) % WORK_GROUPS + WORK_GROUPS) % WORK_GROUPS);
      // raw f16 bits: nothing consumes a prefetched load before its use, so it stays in flight
      unsigned short sraw[4] = {0, 0, 0, 0};
      if (kb < num_kb) {
#pragma unroll
        for (int j = 0; j < 4; ++j) sraw[j] = __ldg(sc_row + (kb * BK + 16 * j) / p.group);
      }
      for (; kb < num_kb; kb += WORK_GROUPS) {
        const long long it = it_base + kb;
        const int stage = static_cast<int>(it % STAGES);
        const uint32_t phase = static_cast<uint32_t>((it / STAGES) & 1);
        const unsigned short cur[4] = {sraw[0], sraw[1], sraw[2], sraw[3]};
        if (kb + WORK_GROUPS < num_kb) {  // the next stage's scales, in flight meanwhile
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            sraw[j] = __ldg(sc_row + ((kb + WORK_GROUPS) * BK + 16 * j) / p.group);
          }
        }
        if (!mbar_wait(&full[stage], phase, abort_flag, p.status, SITE_CONV)) {
          ok = false;
          break;
        }
        // the row's 32 bytes: rows r and r + 4 read their halves in opposite order, so the
        // eight rows of a 128-byte wavefront hit distinct banks
        const uint8_t* qrow = smem + Layout::OFF_Q + stage * Layout::Q_BYTES + n_local * (BK / 2);
        const int sw = (n_local >> 2) & 1;
        const uint4 u0 = *reinterpret_cast<const uint4*>(qrow + 16 * sw);
        const uint4 u1 = *reinterpret_cast<const uint4*>(qrow + 16 * (sw ^ 1));
        const uint4 in0 = sw ? u1 : u0;
        const uint4 in1 = sw ? u0 : u1;
        const uint32_t w[8] = {in0.x, in0.y, in0.z, in0.w, in1.x, in1.y, in1.z, in1.w};
        uint32_t o[32];  // 64 f16 in k order, packed in pairs
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          uint32_t v[4];
          const uint32_t s2 = static_cast<uint32_t>(cur[i / 2]) * 0x10001u;  // (s, s)
          if constexpr (E2M1) {
            e2m1x8_to_f16(w[i], s2, v);
          } else {
            int4x8_to_f16(w[i], s2, v);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) o[4 * i + j] = v[j];
        }
        tmem_st_32x32b_x32(t_lane + static_cast<uint32_t>(TMEM_B_COL + stage * (BK / 2)), o);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[stage]);
      }
      if (!ok) break;
      it_base += num_kb;
      // drain: this warp's 64 columns (m) of D for its 32 rows (n); lanes n (even) and n + 1
      // swap halves so that each stores an (n, n + 1) pair of one row of C
      if (!mbar_wait(tfull, acc_phase, abort_flag, p.status, SITE_EPI)) break;
      tc_fence_after();
      const int n_pair = nb * BN + (n_local & ~1);
      const int c0 = g * (MT_MAX / WORK_GROUPS);
      if (c0 < mt) {
        uint32_t r[2][32];
        tmem_ld_32x32b_x32(t_lane + c0, r[0]);
        if (c0 + 32 < mt) tmem_ld_32x32b_x32(t_lane + c0 + 32, r[1]);
        tmem_ld_wait();
        reg_fence(r[0]);
        reg_fence(r[1]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int m0 = mb * mt + c0 + 32 * h;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float mine_even = __uint_as_float(r[h][2 * i]);
            const float mine_odd = __uint_as_float(r[h][2 * i + 1]);
            const float other = __shfl_xor_sync(0xffffffffu, odd ? mine_even : mine_odd, 1);
            // even lane: row m0 + 2i, (n, n + 1); odd lane: row m0 + 2i + 1, (n - 1, n)
            const int m = m0 + 2 * i + (odd ? 1 : 0);
            const __half2 hv = odd ? __floats2half2_rn(other, mine_odd)
                                   : __floats2half2_rn(mine_even, other);
            if (c0 + 32 * h < mt && m < p.M && n_pair < p.N) {
              *reinterpret_cast<__half2*>(p.c + static_cast<long long>(m) * p.N + n_pair) = hv;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty);
      acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
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
  // m tile = the MMA's N: 256, or M rounded up to 16 when one tile covers M
  const int mt = M >= MT_MAX ? MT_MAX : (M + 15) / 16 * 16;
  CUtensorMap ta, tq;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {BK, static_cast<uint32_t>(mt)};
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
  prm.m_tile = mt;
  prm.status = device_status_ptr();
  auto kernel = dq_gemm_kernel<E2M1>;
  s = set_kernel_smem(reinterpret_cast<const void*>(kernel), Layout::ALLOC);
  if (s != KTA_OK) return s;
  const int tiles = ((M + mt - 1) / mt) * ((N + BN - 1) / BN);
  const int grid = std::max(1, std::min(tiles, current_sm_count()));
  return launch_ex(kernel, dim3(grid), dim3(NUM_THREADS), Layout::ALLOC,
                   static_cast<cudaStream_t>(stream_v), 1, ta, tq, prm);
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
