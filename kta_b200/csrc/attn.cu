// Causal attention forward on the 5th-generation tensor cores (tcgen05), sm_100a.
//
//   O = softmax(Q K^T * scale + causal mask) V,  LSE = logsumexp (natural log, fp32)
//
// It replaces KTA's TileLang fa_forward (perfmodel/testset/gen.py:417-486: online softmax in
// exp2 form with the log2(e)-folded scale, :433, :468-472), made causal, bf16, with the LSE
// output. B200-first design:
//
//   * work unit = (batch, head, 128-row query tile); a persistent grid walks the units
//     head-major (the 32 query tiles of a head run at the same time on different SMs, so
//     that head's K and V are read from HBM once and then served from L2) in a snake order
//     that balances the causal triangle to ~1%;
//   * warp 0: TMA producer (4-D maps over [B, S, H, D], 128-byte swizzle; Q once per unit,
//     K/V tiles through a 2-stage ring); warp 1: TMEM owner and single-thread MMA issuer;
//     warps 2-5: softmax, O correction and epilogue (thread = query row = TMEM lane);
//   * S_j = Q K_j^T lands in one of two TMEM buffers so the tensor core computes S_{j+1}
//     while the softmax warps work on S_j; P_j (bf16) goes to 128-byte-swizzled shared memory
//     as the A operand of O += P_j V_j, with V fed as an MN-major operand; O stays in TMEM;
//   * online softmax with conditional rescaling: the running row maximum used for the
//     exponentials only moves when the true maximum grew by more than 2^8, so O and the row
//     sum are corrected rarely; the final division by the row sum is exact either way;
//   * the causal mask is applied on the diagonal tile only; ragged S is handled by the
//     maps' zero fill (loads) and clipping (stores);
//   * every mbarrier wait is bounded.
#include <algorithm>
#include <cmath>

#include "kta_common.cuh"
#include "kta_host.h"

namespace kta {
namespace attn {

constexpr int D = 128;
constexpr int BM = 128;                 // query rows per unit
constexpr int BN = 128;                 // KV rows per tile
constexpr int NUM_THREADS = 192;        // producer, MMA, 4 softmax warps
constexpr int KV_STAGES = 2;
constexpr int HALF = 128 * 64 * 2;      // [128 rows][64 d] bf16, one swizzle column
constexpr int TILE = 2 * HALF;          // [128 rows][128 d]
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units: rescale when the max grew > 2^8

enum : unsigned int {
  SITE_PROD_Q = 0x401,
  SITE_PROD_KV = 0x402,
  SITE_MMA_Q = 0x403,
  SITE_MMA_K = 0x404,
  SITE_MMA_SFREE = 0x405,
  SITE_MMA_P = 0x406,
  SITE_MMA_V = 0x407,
  SITE_SM_S = 0x408,
  SITE_SM_O = 0x409,
  SITE_EPI_FULL = 0x40a,
  SITE_EPI_FREE = 0x40b,
};

struct Layout {
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + TILE;
  static constexpr int OFF_V = OFF_K + KV_STAGES * TILE;
  static constexpr int OFF_P = OFF_V + KV_STAGES * TILE;  // P tile, then the O staging tile
  static constexpr int OFF_BAR = OFF_P + TILE;
  // q_full, q_empty, k_full[S], v_full[S], kv_empty[S], s_full[2], s_free[2], p_full, o_done,
  // epi_full, epi_free
  static constexpr int NUM_BARS = 2 + 3 * KV_STAGES + 4 + 2 + 2;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int TOTAL = OFF_MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;
  static_assert(ALLOC <= 232448, "shared memory budget of one sm_100 CTA");
};

struct Params {
  float* lse;          // [B, H, S]
  int batch, heads, seq;
  int q_tiles;         // ceil(S / 128)
  float scale_log2;    // softmax scale * log2(e)
  unsigned int* status;
};

__device__ __forceinline__ void tma_load_4d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int32_t x, int32_t y, int32_t z, int32_t w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int32_t x,
                                             int32_t y, int32_t z, int32_t w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

struct Unit {
  int b, h, qt;
};

// Unit index u (head-major, heaviest query tile first within a head).
__device__ __forceinline__ Unit unit_of(int u, const Params& p) {
  Unit r;
  const int bh = u / p.q_tiles;
  r.qt = p.q_tiles - 1 - (u - bh * p.q_tiles);
  r.b = bh / p.heads;
  r.h = bh - r.b * p.heads;
  return r;
}

// The k-th unit of CTA c in the snake order over rounds of gridDim.x units.
__device__ __forceinline__ int snake(int k, int c, int g) {
  return k * g + ((k & 1) ? (g - 1 - c) : c);
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                    const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Layout::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;
  uint64_t* v_full = k_full + KV_STAGES;
  uint64_t* kv_empty = v_full + KV_STAGES;
  uint64_t* s_full = kv_empty + KV_STAGES;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* o_done = p_full + 1;
  uint64_t* epi_full = o_done + 1;  // softmax warps -> storing thread: O staged in smem
  uint64_t* epi_free = epi_full + 1;  // storing thread -> softmax warps: staging read
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Layout::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Layout::OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_init(epi_full, 4);
    mbar_init(epi_free, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);  // S0 [0,128), S1 [128,256), O [256,384)
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int num_units = p.batch * p.heads * p.q_tiles;
  const int rounds = (num_units + gridDim.x - 1) / gridDim.x;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, qphase = 0;
      bool ok = true;
      for (int k = 0; k < rounds && ok; ++k) {
        const int u = snake(k, blockIdx.x, gridDim.x);
        if (u >= num_units) continue;
        const Unit un = unit_of(u, p);
        // Q of this unit once the previous unit's S MMAs are done with the buffer
        if (!mbar_wait(q_empty, qphase ^ 1u, abort_flag, p.status, SITE_PROD_Q)) break;
        qphase ^= 1u;
        mbar_arrive_expect_tx(q_full, TILE);
        tma_load_4d(&tmQ, q_full, smem + Layout::OFF_Q, 0, un.h, un.qt * BM, un.b);
        tma_load_4d(&tmQ, q_full, smem + Layout::OFF_Q + HALF, 64, un.h, un.qt * BM, un.b);
        for (int j = 0; j <= un.qt; ++j) {
          if (!mbar_wait(&kv_empty[stage], phase ^ 1u, abort_flag, p.status, SITE_PROD_KV)) {
            ok = false;
            break;
          }
          uint8_t* kb = smem + Layout::OFF_K + stage * TILE;
          uint8_t* vb = smem + Layout::OFF_V + stage * TILE;
          mbar_arrive_expect_tx(&k_full[stage], TILE);
          tma_load_4d(&tmK, &k_full[stage], kb, 0, un.h, j * BN, un.b);
          tma_load_4d(&tmK, &k_full[stage], kb + HALF, 64, un.h, j * BN, un.b);
          mbar_arrive_expect_tx(&v_full[stage], TILE);
          tma_load_4d(&tmV, &v_full[stage], vb, 0, un.h, j * BN, un.b);
          tma_load_4d(&tmV, &v_full[stage], vb + HALF, 64, un.h, j * BN, un.b);
          if (++stage == KV_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc(BM, BN, 1u, 1u, 0u, 0u);  // Q K^T, both K-major
      constexpr uint32_t idesc_o = make_idesc(BM, D, 1u, 1u, 0u, 1u);   // P V, V MN-major
      const uint32_t q0 = smem_u32(smem + Layout::OFF_Q);
      const uint32_t p0 = smem_u32(smem + Layout::OFF_P);
      const uint32_t t_o = tmem + 256;
      uint32_t kv_t = 0;  // KV tiles this CTA consumed before the current unit
      uint32_t qphase = 0;
      uint32_t sfree_phase[2] = {0, 0};
      uint32_t pphase = 0;
      int s_uses[2] = {0, 0};
      bool ok = true;
      for (int k = 0; k < rounds && ok; ++k) {
        const int u = snake(k, blockIdx.x, gridDim.x);
        if (u >= num_units) continue;
        const Unit un = unit_of(u, p);
        if (!mbar_wait(q_full, qphase, abort_flag, p.status, SITE_MMA_Q)) break;
        qphase ^= 1u;
        tc_fence_after();
        for (int j = 0; j <= un.qt + 1 && ok; ++j) {
          if (j <= un.qt) {
            // ---- S_j = Q K_j^T into S[j & 1] ----
            const int sb = j & 1;
            const uint32_t t = kv_t + static_cast<uint32_t>(j);
            const int st = static_cast<int>(t % KV_STAGES);
            if (!mbar_wait(&k_full[st], (t / KV_STAGES) & 1u, abort_flag, p.status,
                           SITE_MMA_K)) {
              ok = false;
              break;
            }
            if (s_uses[sb] > 0) {
              if (!mbar_wait(&s_free[sb], sfree_phase[sb], abort_flag, p.status,
                             SITE_MMA_SFREE)) {
                ok = false;
                break;
              }
              sfree_phase[sb] ^= 1u;
            }
            ++s_uses[sb];
            tc_fence_after();
            const uint32_t k0 = smem_u32(smem + Layout::OFF_K + st * TILE);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk >> 2) * HALF + (kk & 3) * 32;
              umma_f16(tmem + sb * BN, sdesc_sw128(q0 + off, 16, 1024),
                       sdesc_sw128(k0 + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
            }
            umma_commit(&s_full[sb]);
            if (j == un.qt) umma_commit(q_empty);  // the unit's last read of Q
          }
          if (j >= 1) {
            // ---- O += P_{j-1} V_{j-1} ----
            if (!mbar_wait(p_full, pphase, abort_flag, p.status, SITE_MMA_P)) {
              ok = false;
              break;
            }
            pphase ^= 1u;
            const uint32_t t = kv_t + static_cast<uint32_t>(j - 1);
            const int st = static_cast<int>(t % KV_STAGES);
            if (!mbar_wait(&v_full[st], (t / KV_STAGES) & 1u, abort_flag, p.status,
                           SITE_MMA_V)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t v0 = smem_u32(smem + Layout::OFF_V + st * TILE);
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk) {
              const uint32_t aoff = (kk >> 2) * HALF + (kk & 3) * 32;
              umma_f16(t_o, sdesc_sw128(p0 + aoff, 16, 1024),
                       sdesc_sw128(v0 + kk * 16 * 128, HALF, 1024), idesc_o,
                       (j - 1 > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(o_done);
            umma_commit(&kv_empty[st]);
          }
        }
        kv_t += static_cast<uint32_t>(un.qt + 1);
      }
    }
  } else {
    // ---------------- softmax, O correction and epilogue (thread = query row) ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    uint8_t* pbuf = smem + Layout::OFF_P;
    uint32_t sfull_phase[2] = {0, 0};
    uint32_t ophase = 0;
    uint32_t ephase = 0;
    bool ok = true;
    for (int k = 0; k < rounds && ok; ++k) {
      const int u = snake(k, blockIdx.x, gridDim.x);
      if (u >= num_units) continue;
      const Unit un = unit_of(u, p);
      float m_used = -INFINITY;  // log2-domain maximum the exponentials are relative to
      float lsum = 0.f;
      for (int j = 0; j <= un.qt; ++j) {
        const int sb = j & 1;
        if (!mbar_wait(&s_full[sb], sfull_phase[sb], abort_flag, p.status, SITE_SM_S)) {
          ok = false;
          break;
        }
        sfull_phase[sb] ^= 1u;
        tc_fence_after();
        float s[BN];
#pragma unroll
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem + lane_base + sb * BN + c, r);
          tmem_ld_wait();
          reg_fence(r);
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c + i] = __uint_as_float(r[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[sb]);
        // scale into the log2 domain, causal mask on the diagonal tile
        const bool diag = (j == un.qt);
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          float v = s[c] * p.scale_log2;
          if (diag && c > row) v = -INFINITY;
          s[c] = v;
          mx = fmaxf(mx, v);
        }
        float factor = 1.f;
        bool rescale = false;
        if (mx > m_used + RESCALE_THRESHOLD || m_used == -INFINITY) {
          const float m_new = fmaxf(mx, m_used);
          factor = (m_used == -INFINITY) ? 0.f : exp2f(m_used - m_new);
          rescale = m_used != -INFINITY;
          m_used = m_new;
        }
        float rs = 0.f;
        uint32_t pk[BN / 2];
#pragma unroll
        for (int c = 0; c < BN; c += 2) {
          const float e0 = (m_used == -INFINITY) ? 0.f : exp2f(s[c] - m_used);
          const float e1 = (m_used == -INFINITY) ? 0.f : exp2f(s[c + 1] - m_used);
          rs += e0 + e1;
          pk[c / 2] = pack_bf16x2(e0, e1);
        }
        lsum = lsum * factor + rs;
        // PV_{j-1} must be complete before P is overwritten and before O is corrected
        if (j >= 1) {
          if (!mbar_wait(o_done, ophase, abort_flag, p.status, SITE_SM_O)) {
            ok = false;
            break;
          }
          ophase ^= 1u;
          tc_fence_after();
          if (__any_sync(0xffffffffu, rescale)) {
            const float f = rescale ? factor : 1.f;
#pragma unroll
            for (int c = 0; c < D; c += 16) {
              uint32_t r[16];
              tmem_ld_32x32b_x16(tmem + lane_base + 256 + c, r);
              tmem_ld_wait();
              reg_fence(r);
#pragma unroll
              for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * f);
              tmem_st_32x32b_x16(tmem + lane_base + 256 + c, r);
            }
            tmem_st_wait();
          }
        }
        // P row -> 128-byte-swizzled K-major A operand: row `row`, two 64-wide halves
        {
          const uint32_t base = smem_u32(pbuf) + static_cast<uint32_t>(row) * 128u;
#pragma unroll
          for (int c8 = 0; c8 < BN / 8; ++c8) {
            const uint32_t half = static_cast<uint32_t>(c8 >> 3) * HALF;
            const uint32_t chunk = static_cast<uint32_t>((c8 & 7) ^ (row & 7));
            st_shared_v4(base + half + (chunk << 4), pk[c8 * 4], pk[c8 * 4 + 1], pk[c8 * 4 + 2],
                         pk[c8 * 4 + 3]);
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
      }
      if (!ok) break;
      // ---- epilogue: O / l -> bf16 -> smem (P buffer) -> TMA store; LSE ----
      if (!mbar_wait(o_done, ophase, abort_flag, p.status, SITE_SM_O)) break;
      ophase ^= 1u;
      tc_fence_after();
      const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
      {
        const uint32_t base = smem_u32(pbuf) + static_cast<uint32_t>(row) * 128u;
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem + lane_base + 256 + c, r);
          tmem_ld_wait();
          reg_fence(r);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            pk[i] = pack_bf16x2(__uint_as_float(r[2 * i]) * inv, __uint_as_float(r[2 * i + 1]) * inv);
          }
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            const int cc = c / 8 + c8;  // 16-byte chunk index 0..15 along d
            const uint32_t half = static_cast<uint32_t>(cc >> 3) * HALF;
            const uint32_t chunk = static_cast<uint32_t>((cc & 7) ^ (row & 7));
            st_shared_v4(base + half + (chunk << 4), pk[c8 * 4], pk[c8 * 4 + 1], pk[c8 * 4 + 2],
                         pk[c8 * 4 + 3]);
          }
        }
      }
      const int qrow = un.qt * BM + row;
      if (qrow < p.seq) {
        const float lse = lsum > 0.f ? (m_used + __log2f(lsum)) * 0.6931471805599453f : -INFINITY;
        p.lse[(static_cast<long long>(un.b) * p.heads + un.h) * p.seq + qrow] = lse;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(epi_full);
      if (threadIdx.x == 64) {
        // all four softmax warps staged their O rows: store the tile
        if (mbar_wait(epi_full, ephase, abort_flag, p.status, SITE_EPI_FULL)) {
          tma_store_4d(&tmO, pbuf, 0, un.h, un.qt * BM, un.b);
          tma_store_4d(&tmO, pbuf + HALF, 64, un.h, un.qt * BM, un.b);
          bulk_commit_group();
          bulk_wait_group_read<0>();  // the P buffer is reused by the next unit
        }
        mbar_arrive(epi_free);
      }
      if (!mbar_wait(epi_free, ephase, abort_flag, p.status, SITE_EPI_FREE)) break;
      ephase ^= 1u;
    }
    if (threadIdx.x == 64) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int launch(const void* Q, const void* K, const void* V, void* O, void* LSE, int64_t B,
           int64_t H, int64_t S, int64_t Dm, float scale, cudaStream_t stream) {
  if (!Q || !K || !V || !O || !LSE) return KTA_ERR_INVALID_ARG;
  if (B <= 0 || H <= 0 || S <= 0) return KTA_ERR_INVALID_ARG;
  if (!(scale > 0.f) || !std::isfinite(scale)) return KTA_ERR_INVALID_ARG;
  if (Dm != D) return KTA_ERR_UNSUPPORTED;
  if (B > 65535 || H > 65535 || S > (1 << 24) || B * H * ((S + BM - 1) / BM) > (1LL << 31) - 1) {
    return KTA_ERR_UNSUPPORTED;
  }
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O) ||
      (reinterpret_cast<uintptr_t>(LSE) & 3)) {
    return KTA_ERR_ALIGN;
  }
  int s = require_sm100();
  if (s != KTA_OK) return s;
  // [B, S, H, D] as a 4-D map: d innermost, then h, s, b
  const uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(H),
                            static_cast<uint64_t>(S), static_cast<uint64_t>(B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(H * D) * 2,
                               static_cast<uint64_t>(S * H * D) * 2};
  const uint32_t box[4] = {64, 1, 128, 1};
  CUtensorMap tq, tk, tv, to;
  const void* ptrs[4] = {Q, K, V, O};
  CUtensorMap* maps[4] = {&tq, &tk, &tv, &to};
  for (int i = 0; i < 4; ++i) {
    s = encode_tmap(maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, ptrs[i], dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  Params prm;
  prm.lse = static_cast<float*>(LSE);
  prm.batch = static_cast<int>(B);
  prm.heads = static_cast<int>(H);
  prm.seq = static_cast<int>(S);
  prm.q_tiles = static_cast<int>((S + BM - 1) / BM);
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.status = device_status_ptr();
  s = set_kernel_smem(reinterpret_cast<const void*>(attn_fwd_kernel), Layout::ALLOC);
  if (s != KTA_OK) return s;
  const long long units = B * H * static_cast<long long>(prm.q_tiles);
  const int grid = static_cast<int>(std::max(1LL, std::min<long long>(current_sm_count(), units)));
  attn_fwd_kernel<<<grid, NUM_THREADS, Layout::ALLOC, stream>>>(tq, tk, tv, to, prm);
  return launch_status();
}

}  // namespace attn
}  // namespace kta

extern "C" int kta_attn_fwd_causal_bf16(const void* Q, const void* K, const void* V, void* O,
                                        void* LSE, int64_t B, int64_t H, int64_t S, int64_t D,
                                        float scale, void* stream) {
  return kta::attn::launch(Q, K, V, O, LSE, B, H, S, D, scale, static_cast<cudaStream_t>(stream));
}
