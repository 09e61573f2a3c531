// GEMM C = A·Bᵀ for M <= 16 (the decode-time "skinny" case, e.g. 16 x 8192 x 8192), sm_100a.
//
// HBM-bound on B (N x K): the job is to stream B once at full bandwidth on every SM. The
// tensor-memory kernels tile N by 128 (UMMA M), and 148 SMs do not divide a power-of-two N
// into 128-row tiles: 8192 rows give 64 tiles, so a K split can only fill 128 SMs. Here the
// contraction runs on mma.sync m16n8k16 with the roles of the reference statement kept:
// M = 16 rows of A on the MMA's M, 8 rows of B per n8 tile. N is cut into n8 tiles and every
// CTA of a one-wave grid takes a contiguous run of NT (<= 8) of them over the whole of K, so
// all SMs stream, no partial sums cross CTAs and the result is deterministic.
//
//   * warp 0: TMA producer; per stage four 64-wide K boxes of B (8·NT rows, 128-byte
//     swizzle: each row is fetched as one 512-byte run) and of A (16 rows), 5-6 stage ring;
//   * warps 1-8: each owns 32 of the stage's 256 K columns: ldmatrix of A (16x16) and of the
//     NT n8 tiles of B, mma.sync into NT x 4 fp32 accumulators; one release per stage;
//   * the eight per-warp partials are summed through shared memory and stored as C rows.
//
// Algorithmic bytes per launch: (M·K + N·K + M·N)·2, FLOP 2·M·N·K. Every mbarrier wait is
// bounded.
#include <algorithm>
#include <type_traits>

#include "kta_common.cuh"
#include "kta_host.h"

namespace kta {
namespace gemm {

namespace m16 {

constexpr int THREADS = 288;  // producer warp + 8 compute warps
constexpr int COMPUTE_WARPS = 8;
constexpr int BOX_K = 64;     // one 128-byte swizzle row of 16-bit elements
constexpr int SUB = 4;        // boxes per stage
constexpr int STAGE_K = SUB * BOX_K;

enum : unsigned int {
  SITE_EMPTY = 0x601,
  SITE_FULL = 0x602,
};

template <int NT>
struct Layout {
  static constexpr int B_BOX = 8 * NT * BOX_K * 2;      // 8·NT rows x 128 B
  static constexpr int A_BOX = 16 * BOX_K * 2;          // 16 rows x 128 B
  static_assert(B_BOX % 1024 == 0, "swizzled boxes start on 1024-byte boundaries");
  static constexpr int STAGE_BYTES = SUB * (B_BOX + A_BOX);
  static constexpr int FIT = (232448 - 2048) / STAGE_BYTES;
  static constexpr int STAGES = FIT < 6 ? FIT : 6;  // 6 stages (216 KB) for NT = 7
  static constexpr int OFF_BAR = STAGES * STAGE_BYTES;
  static constexpr int OFF_MISC = OFF_BAR + 2 * STAGES * 8;
  static constexpr int TOTAL = OFF_MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;
  // per-warp partials [warp][16][8·NT] fp32, over the stage ring once the main loop is done
  static_assert(COMPUTE_WARPS * 16 * 8 * NT * 4 <= STAGES * STAGE_BYTES, "reduction area");
  static_assert(ALLOC <= 232448, "shared memory budget of one sm_100 CTA");
};

__device__ __forceinline__ uint32_t swz(uint32_t base, int row, int chunk) {
  return base + static_cast<uint32_t>(row) * 128u +
         (static_cast<uint32_t>(chunk ^ (row & 7)) << 4);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

template <bool BF16>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32"
        " {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32"
        " {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ void compute_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(COMPUTE_WARPS * 32) : "memory");
}

// CTA c owns n8 tiles [c·NT, c·NT + NT) ∩ [0, tiles8).
template <int NT, bool BF16>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_m16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    void* __restrict__ Cv, int M, int N, int K, int64_t ldc, int prefetch,
                    unsigned int* status) {
  using L = Layout<NT>;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + L::STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC);

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * NT * 8;  // first row of B (column of C) of this CTA
  const int num_stages = (K + STAGE_K - 1) / STAGE_K;

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], COMPUTE_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  __syncthreads();
  pdl_launch_dependents();
  if (prefetch && warp == 0 && lane == 0) {
    // While the previous grid finishes, pull the boxes of the first ring's worth of stages
    // into L2, so the stream does not start with a full HBM round trip after the wait.
    const int pre = num_stages < L::STAGES ? num_stages : L::STAGES;
    for (int ks = 0; ks < pre; ++ks) {
#pragma unroll
      for (int u = 0; u < SUB; ++u) {
        tma_prefetch_l2_2d(&tmB, ks * STAGE_K + u * BOX_K, row0);
        if (blockIdx.x == 0) tma_prefetch_l2_2d(&tmA, ks * STAGE_K + u * BOX_K, 0);
      }
    }
  }
  pdl_wait();  // the previous grid's writes (this launch's inputs) are visible from here on

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int ks = 0; ks < num_stages; ++ks) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status, SITE_EMPTY)) break;
        uint8_t* st = smem + stage * L::STAGE_BYTES;
        // full boxes are counted even where the tensor's edge zero-fills them
        mbar_arrive_expect_tx(&full[stage], L::STAGE_BYTES);
#pragma unroll
        for (int u = 0; u < SUB; ++u) {
          tma_load_2d(&tmB, &full[stage], st + u * L::B_BOX, ks * STAGE_K + u * BOX_K, row0);
        }
#pragma unroll
        for (int u = 0; u < SUB; ++u) {
          tma_load_2d(&tmA, &full[stage], st + SUB * L::B_BOX + u * L::A_BOX,
                      ks * STAGE_K + u * BOX_K, 0);
        }
        if (++stage == L::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    return;  // the producer takes no part in the reduction below
  }

  // ---- compute warps: warp w owns K columns [32w, 32w + 32) of every stage ----
  const int w = warp - 1;
  const int box = w >> 1;               // which 64-wide box of the stage
  const int chunk0 = (w & 1) * 4;       // first 16-byte chunk (8 columns) inside the box
  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[t][i] = 0.f;
  }
  int stage = 0;
  uint32_t phase = 0;
  bool ok = true;
  for (int ks = 0; ks < num_stages; ++ks) {
    if (!mbar_wait(&full[stage], phase, abort_flag, status, SITE_FULL)) {
      ok = false;
      break;
    }
    const uint32_t st = smem_u32(smem + stage * L::STAGE_BYTES);
    const uint32_t bbase = st + box * L::B_BOX;
    const uint32_t abase = st + SUB * L::B_BOX + box * L::A_BOX;
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int c = chunk0 + 2 * s;
      uint32_t a[4];
      ldsm_x4(swz(abase, lane & 15, c + (lane >> 4)), a);
#pragma unroll
      for (int t = 0; t + 1 < NT; t += 2) {
        uint32_t b[4];
        ldsm_x4(swz(bbase, t * 8 + (lane & 7) + ((lane >> 4) << 3), c + ((lane >> 3) & 1)), b);
        mma16816<BF16>(acc[t], a, b[0], b[1]);
        mma16816<BF16>(acc[t + 1], a, b[2], b[3]);
      }
      if constexpr (NT % 2 == 1) {
        uint32_t b0, b1;
        ldsm_x2(swz(bbase, (NT - 1) * 8 + (lane & 7), c + ((lane >> 3) & 1)), b0, b1);
        mma16816<BF16>(acc[NT - 1], a, b0, b1);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == L::STAGES) {
      stage = 0;
      phase ^= 1u;
    }
  }

  // ---- reduction of the eight partials; the ring is free once every warp passed its loop
  // (each waited for every stage's bytes) ----
  compute_bar();
  float* red = reinterpret_cast<float*>(smem);  // [8][16][8·NT]
  constexpr int W = 8 * NT;
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    float* p = red + (w * 16) * W + t * 8 + 2 * q;
    p[g * W] = acc[t][0];
    p[g * W + 1] = acc[t][1];
    p[(g + 8) * W] = acc[t][2];
    p[(g + 8) * W + 1] = acc[t][3];
  }
  compute_bar();
  if (!ok || *abort_flag) return;
  T* C = reinterpret_cast<T*>(Cv);
  for (int e = threadIdx.x - 32; e < 16 * W; e += COMPUTE_WARPS * 32) {
    const int m = e / W, n = e - m * W;
    float v = 0.f;
#pragma unroll
    for (int k = 0; k < COMPUTE_WARPS; ++k) v += red[k * 16 * W + e];
    const int col = row0 + n;
    if (m < M && col < N) {
      if constexpr (BF16) {
        C[static_cast<int64_t>(m) * ldc + col] = __float2bfloat16_rn(v);
      } else {
        C[static_cast<int64_t>(m) * ldc + col] = __float2half_rn(v);
      }
    }
  }
}

template <int NT, bool BF16>
int launch_nt(const void* A, const void* B, void* C, int M, int N, int K, int64_t lda,
              int64_t ldb, int64_t ldc, cudaStream_t stream) {
  using L = Layout<NT>;
  const CUtensorMapDataType dt =
      BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(lda) * 2};
    const uint32_t box[2] = {BOX_K, 16};
    int s = encode_tmap(&ta, dt, 2, A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldb) * 2};
    const uint32_t box[2] = {BOX_K, static_cast<uint32_t>(8 * NT)};
    int s = encode_tmap(&tb, dt, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  auto kernel = gemm_m16_kernel<NT, BF16>;
  int s = set_kernel_smem(reinterpret_cast<const void*>(kernel), L::ALLOC);
  if (s != KTA_OK) return s;
  const int tiles8 = (N + 7) / 8;
  const int grid = (tiles8 + NT - 1) / NT;
  const int prefetch = static_cast<int64_t>(N) * K * 2 > kPrefetchMinBytes ? 1 : 0;
  return launch_ex(kernel, dim3(grid), dim3(THREADS), L::ALLOC, stream, 1, ta, tb, C, M, N, K,
                   ldc, prefetch, device_status_ptr());
}

}  // namespace m16

// M <= 16, B K-major. Returns KTA_ERR_UNSUPPORTED when N needs more than one wave of CTAs
// with 8 n8 tiles each (the caller then uses the tensor-memory kernel).
template <bool BF16>
int launch_m16(const void* A, const void* B, void* C, int M, int N, int K, int64_t lda,
               int64_t ldb, int64_t ldc, cudaStream_t stream) {
  if (M > 16) return KTA_ERR_UNSUPPORTED;
  const int sms = std::max(1, current_sm_count());
  const int tiles8 = (N + 7) / 8;
  const int nt = (tiles8 + sms - 1) / sms;  // n8 tiles per CTA for one wave
  switch (nt) {
    case 1: return m16::launch_nt<1, BF16>(A, B, C, M, N, K, lda, ldb, ldc, stream);
    case 2: return m16::launch_nt<2, BF16>(A, B, C, M, N, K, lda, ldb, ldc, stream);
    case 3: return m16::launch_nt<3, BF16>(A, B, C, M, N, K, lda, ldb, ldc, stream);
    case 4: return m16::launch_nt<4, BF16>(A, B, C, M, N, K, lda, ldb, ldc, stream);
    case 5: return m16::launch_nt<5, BF16>(A, B, C, M, N, K, lda, ldb, ldc, stream);
    case 6: return m16::launch_nt<6, BF16>(A, B, C, M, N, K, lda, ldb, ldc, stream);
    case 7: return m16::launch_nt<7, BF16>(A, B, C, M, N, K, lda, ldb, ldc, stream);
    case 8: return m16::launch_nt<8, BF16>(A, B, C, M, N, K, lda, ldb, ldc, stream);
    default: return KTA_ERR_UNSUPPORTED;
  }
}

template int launch_m16<true>(const void*, const void*, void*, int, int, int, int64_t, int64_t,
                              int64_t, cudaStream_t);
template int launch_m16<false>(const void*, const void*, void*, int, int, int, int64_t, int64_t,
                               int64_t, cudaStream_t);

}  // namespace gemm
}  // namespace kta
