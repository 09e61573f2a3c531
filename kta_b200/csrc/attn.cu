// Causal attention forward on the 5th-generation tensor cores (tcgen05), sm_100a.
//
//   O = softmax(Q K^T * scale + causal mask) V,  LSE = logsumexp (natural log, fp32)
//
// It replaces KTA's TileLang fa_forward (perfmodel/testset/gen.py:417-486: online softmax in
// exp2 form with the log2(e)-folded scale, :433, :468-472), made causal, bf16, with the LSE
// output. B200-first design:
//
//   * work unit = (batch, head, a pair of 128-row query tiles A and B); a persistent grid
//     walks the units head-major (the query tiles of one head run at the same time on
//     different SMs, so that head's K and V come from HBM once and then from L2), heaviest
//     pair first, in a snake order that balances the causal triangle; when every head's K
//     and V fit in L2 together (one GPU's share of a sharded batch), cost-major instead;
//   * three warpgroups: warps 0-3 and 4-7 are the softmax warpgroups of tiles A and B
//     (thread = query row = TMEM lane); in the third, warp 8 is the TMA producer of Q_A and
//     K (2-stage ring), warp 9 the TMEM owner and MMA issuer (the warp walks the schedule,
//     one elected lane issues), warp 10 the TMA producer of Q_B and V (2-stage ring), warp 11
//     idle; each Q tile has its own barriers and is loaded as soon as the unit's last S of
//     that tile has read the previous one; all loads go through 4-D
//     maps over [B, S, H, D] with 128-byte swizzle. setmaxnreg moves registers from the
//     third warpgroup (88 per thread) to the softmax ones (208), which hold a whole S row;
//   * TMEM: S_A, S_B (128 columns each), O_A, O_B (128 each). P (bf16) is written back over
//     the first 64 columns of its S and read by O += P V straight from TMEM (A operand in
//     tensor memory, V as an MN-major shared-memory operand): no shared-memory round trip;
//   * MMA order per KV tile j: S_A(j), PV_B(j-1), S_B(j), PV_A(j): while one warpgroup turns
//     S into P the tensor core works for the other; tcgen05 ops of one thread complete in
//     order, so "S(j) done" also means "PV(j-1) done" for the same tile. The softmax
//     publishes P in two halves (keys 0-63, 64-127) and PV starts on the first while the
//     second is computed. A unit's last KV step is tile B's alone; when the next unit's Q_A
//     and first K tile have landed by then, its S_A(0) is issued before that step's PV_B, so
//     the tensor core and tile A's softmax work while B's diagonal softmax finishes;
//   * softmax in one pass over a row held in registers: max on raw scores (3-input max),
//     packed f32x2 FFMA for scale-and-subtract, and the exponentials split between the MUFU
//     (ex2.approx.ftz) and the FMA pipe (Cody-Waite reduction 2^x = 2^j 2^f, |f| <= 1/2, with
//     a degree-3 minimax polynomial for 2^f, max relative error 7.5e-5, far below bf16's
//     rounding of P); the running maximum moves only when the true one grew by more than
//     2^8, so O and the row sum are corrected rarely (the final division by the row sum is
//     exact either way); the causal mask is applied on diagonal tiles only, whose
//     exponentials all go to the MUFU (it maps -inf to 0);
//   * every mbarrier wait is bounded.
#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "kta_common.cuh"
#include "kta_host.h"

namespace kta {
namespace attn {

constexpr int D = 128;
constexpr int BM = 128;                 // query rows per tile
constexpr int BN = 128;                 // KV rows per tile
constexpr int NUM_THREADS = 384;        // two softmax warpgroups, producers + MMA warpgroup
constexpr int K_STAGES = 2;
constexpr int V_STAGES = 2;
constexpr int QK_PRODUCER_WARP = 8;
constexpr int MMA_WARP = 9;
constexpr int V_PRODUCER_WARP = 10;
constexpr int SOFTMAX_REGS = 208;       // 2 x 128 x 208 + 128 x 88 = 384 x 168 (launch)
constexpr int OTHER_REGS = 88;
// exponentials evaluated on the FMA pipe, per 8 column pairs of an off-diagonal tile
constexpr int EXP_POLY_PER_8 = 2;
constexpr int HALF = 128 * 64 * 2;      // [128 rows][64 d] bf16, one swizzle column
constexpr int TILE = 2 * HALF;          // [128 rows][128 d]
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units: rescale when the max grew > 2^8

// TMEM columns: S of tile t at t * 128, O of tile t at 256 + t * 128
__host__ __device__ constexpr uint32_t t_s_col(int t) { return static_cast<uint32_t>(t) * 128u; }
__host__ __device__ constexpr uint32_t t_o_col(int t) { return 256u + static_cast<uint32_t>(t) * 128u; }

enum : unsigned int {
  SITE_PROD_Q = 0x401,
  SITE_PROD_KV = 0x402,
  SITE_MMA_Q = 0x403,
  SITE_MMA_K = 0x404,
  SITE_MMA_V = 0x405,
  SITE_MMA_P = 0x406,
  SITE_MMA_OFREE = 0x407,
  SITE_SM_S = 0x408,
  SITE_SM_O = 0x409,
};

struct Layout {
  static constexpr int OFF_Q = 0;                           // Q_A, Q_B
  static constexpr int OFF_K = OFF_Q + 2 * TILE;
  static constexpr int OFF_V = OFF_K + K_STAGES * TILE;
  static constexpr int OFF_BAR = OFF_V + V_STAGES * TILE;
  // q_full[2], q_empty[2] (per query tile), k_full[K], k_empty[K], v_full[V], v_empty[V], s_full[2],
  // p_full[2][2] (tile, half of P), o_done[2], o_free[2]
  static constexpr int NUM_BARS = 4 + 2 * K_STAGES + 2 * V_STAGES + 10;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int TOTAL = OFF_MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;
  static_assert(ALLOC <= 232448, "shared memory budget of one sm_100 CTA");
};

struct Params {
  __nv_bfloat16* out;  // [B, S, H, D]
  float* lse;          // [B, H, S]
  int batch, heads, seq;
  int q_tiles;         // ceil(S / 128)
  int pairs;           // ceil(q_tiles / 2)
  float scale_log2;    // softmax scale * log2(e)
  int tail;            // issue the next unit's first S_A during the last (tile B only) step
  int cost_major;      // unit order by pair (cost) across heads instead of head-major
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

// Non-blocking probe of an mbarrier phase (mbarrier.test_wait): true once it completed.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n"
      " .reg .pred P;\n"
      " mbarrier.test_wait.parity.shared::cta.b64 P, [%1], %2;\n"
      " selp.u32 %0, 1, 0, P;\n"
      "}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n"
      " .reg .pred P;\n"
      " elect.sync _|P, 0xffffffff;\n"
      " selp.b32 %0, 1, 0, P;\n"
      "}\n"
      : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x0, 2^x1 on the FMA pipe for x <= 2^8 (the rescale threshold bounds x from above).
// Cody-Waite: j = round(x) by the 1.5 * 2^23 shifter, f = x - j in [-1/2, 1/2], 2^f from a
// degree-3 polynomial (minimax in relative error, fitted for this kernel: max 7.5e-5), and
// 2^j added into the exponent field. x is clamped at -125 so that 2^j p(f) stays a normal
// number; 2^-125 stands in for smaller results (they vanish against a row sum >= 1).
__device__ __forceinline__ void exp2_poly_pair(uint64_t x, float& e0, float& e1) {
  float x0, x1;
  f2_split(x, x0, x1);
  x = f2(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t shifter = f2(12582912.f, 12582912.f);
  const uint64_t unshift = f2(-12582912.f, -12582912.f);
  const uint64_t t = add2(x, shifter);             // low mantissa bits hold j
  const uint64_t fr = sub2(x, add2(t, unshift));
  uint64_t p = fma2(f2(0.0551716648f, 0.0551716648f), fr, f2(0.242611170f, 0.242611170f));
  p = fma2(p, fr, f2(0.693260968f, 0.693260968f));
  p = fma2(p, fr, f2(0.999928057f, 0.999928057f));
  float p0, p1, t0, t1;
  f2_split(p, p0, p1);
  f2_split(t, t0, t1);
  e0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  e1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

struct Unit {
  int b, h, pair;
  bool has_b;   // the second query tile exists (q_tiles may be odd)
  int nkv;      // KV tiles the unit reads: through tile B's diagonal (or A's)
};

// Unit index u: head-major, heaviest pair first within a head (a head's units run at about
// the same time, so its K and V come from HBM once); or, when every head's K and V fit in L2
// together, cost-major: the heaviest pair of every head first, so the snake over rounds
// balances the CTAs (95.8 % instead of 86.5 % of the ideal for one batch entry of 32 heads).
__device__ __forceinline__ Unit unit_of(int u, const Params& p) {
  Unit r;
  int bh;
  if (p.cost_major) {
    const int nbh = p.batch * p.heads;
    const int lvl = u / nbh;
    bh = u - lvl * nbh;
    r.pair = p.pairs - 1 - lvl;
  } else {
    bh = u / p.pairs;
    r.pair = p.pairs - 1 - (u - bh * p.pairs);
  }
  r.b = bh / p.heads;
  r.h = bh - r.b * p.heads;
  r.has_b = 2 * r.pair + 1 < p.q_tiles;
  r.nkv = r.has_b ? 2 * r.pair + 2 : 2 * r.pair + 1;
  return r;
}

// The k-th unit of CTA c in the snake order over rounds of gridDim.x units.
__device__ __forceinline__ int snake(int k, int c, int g) {
  return k * g + ((k & 1) ? (g - 1 - c) : c);
}

// One softmax step for this thread's query row over a 128-column S tile in TMEM: the row
// maximum (pass 1), the decision to move the running maximum, and P = 2^(s*scale - m) packed
// to bf16 pairs over the S columns already consumed (pass 2). DIAG applies the causal mask
// (key c visible to query `row` iff c <= row); off the diagonal no mask code runs.
// One S tile of one query row (this thread's TMEM lane): P = 2^(S sl - m) as bf16 over the
// first 64 columns, published in two halves (p_half[0], p_half[1]), the running maximum m
// (log2 units) and the row sum l. When m moved, O is rescaled in TMEM before the first half
// is published (PV(j-1) completed before S(j) did: same issuing thread, in order).
template <bool DIAG>
__device__ __forceinline__ void softmax_step(uint32_t t_s, uint32_t t_o, int row, int lane,
                                             float sl, float& m_used, float& lsum,
                                             uint64_t* p_half) {
  uint32_t r[BN];
#pragma unroll
  for (int q = 0; q < BN / 32; ++q) {
    tmem_ld_32x32b_x32(t_s + q * 32, *reinterpret_cast<uint32_t(*)[32]>(r + q * 32));
  }
  tmem_ld_wait();
  reg_fence(r);
  if (DIAG) {
#pragma unroll
    for (int c = 0; c < BN; ++c) {
      if (c > row) r[c] = __float_as_uint(-INFINITY);
    }
  }
  float mx[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
#pragma unroll
  for (int i = 0; i < BN / 2; ++i) {
    mx[i & 7] = max3(mx[i & 7], __uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
  }
  const float rmax = max3(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], mx[5]),
                          fmaxf(mx[6], mx[7])) * sl;
  float factor = 1.f;
  bool rescale = false;
  if (rmax > m_used + RESCALE_THRESHOLD) {
    factor = ex2(m_used - rmax);  // 0 on the first tile (m_used = -inf, lsum = 0)
    rescale = m_used != -INFINITY;
    m_used = rmax;
  }
  lsum *= factor;
  const bool any_rescale = __any_sync(0xffffffffu, rescale);
  const uint64_t sl2 = f2(sl, sl);
  const uint64_t neg2 = f2(-m_used, -m_used);
  uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t pk[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int c = h * 64 + 2 * i;
      const uint64_t x = fma2(f2(__uint_as_float(r[c]), __uint_as_float(r[c + 1])), sl2, neg2);
      float e0, e1;
      if (!DIAG && (i & 7) >= 8 - EXP_POLY_PER_8) {
        exp2_poly_pair(x, e0, e1);
      } else {
        float x0, x1;
        f2_split(x, x0, x1);
        e0 = ex2(x0);
        e1 = ex2(x1);
      }
      sum2[i & 3] = add2(sum2[i & 3], f2(e0, e1));
      pk[i] = pack_bf16x2(e0, e1);
    }
    if (h == 0 && any_rescale) {
      // with half of the row already turned into P, fewer registers are live here
      const float f = rescale ? factor : 1.f;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(t_o + c, o);
        tmem_ld_wait();
        reg_fence(o);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
        tmem_st_32x32b_x32(t_o + c, o);
      }
    }
    tmem_st_32x32b_x32(t_s + h * 32, pk);
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&p_half[h]);
  }
  const uint64_t s01 = add2(add2(sum2[0], sum2[1]), add2(sum2[2], sum2[3]));
  float s0, s1;
  f2_split(s01, s0, s1);
  lsum += s0 + s1;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Layout::OFF_BAR);
  uint64_t* q_full = bars;        // [tile]: Q_A (the QK warp loads it), Q_B (the V warp)
  uint64_t* q_empty = bars + 2;   // [tile]: released by the unit's last S of that tile
  uint64_t* k_full = bars + 4;
  uint64_t* k_empty = k_full + K_STAGES;
  uint64_t* v_full = k_empty + K_STAGES;
  uint64_t* v_empty = v_full + V_STAGES;
  uint64_t* s_full = v_empty + V_STAGES;    // [tile]
  uint64_t* p_full = s_full + 2;            // [tile][half]: P columns of keys 64h..64h+63
  uint64_t* o_done = p_full + 4;            // [tile]: the unit's last PV completed
  uint64_t* o_free = o_done + 2;            // [tile]: the epilogue read O
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Layout::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Layout::OFF_MISC + 4);

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(&q_full[t], 1);
      mbar_init(&q_empty[t], 1);
    }
    for (int s = 0; s < K_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < V_STAGES; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[2 * i], 4);
      mbar_init(&p_full[2 * i + 1], 4);
      mbar_init(&o_done[i], 1);
      mbar_init(&o_free[i], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == QK_PRODUCER_WARP && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_launch_dependents();
  pdl_wait();  // the previous grid's writes (this launch's inputs) are visible from here on
  const int num_units = p.batch * p.heads * p.pairs;
  const int rounds = (num_units + gridDim.x - 1) / gridDim.x;

  // registers move from the producer/MMA warpgroup to the softmax warpgroups; each
  // setmaxnreg dominates the code of its warpgroup
  if (warp >= QK_PRODUCER_WARP) {
    setmaxnreg_dec<OTHER_REGS>();
    if (warp == QK_PRODUCER_WARP || warp == V_PRODUCER_WARP) {
      // ------------------- TMA producers: Q and K (warp 8), V (warp 10) -------------------
      if (lane == 0) {
        const bool is_k = warp == QK_PRODUCER_WARP;
        // the QK warp loads Q_A and K, the V warp Q_B and V: each Q tile is loaded as soon as
        // its slot is free, the other tile's slot may still be in use
        const int qt = is_k ? 0 : 1;
        uint32_t kv_t = 0, qphase = 0;
        bool ok = true;
        // Per unit: the first K (or V) tile, then the Q tile (its slot frees only at the
        // previous unit's last S of that tile), then the remaining tiles, so that the first
        // K / V tile of a unit does not queue behind the wait for the Q slot.
        auto load_kv = [&](const Unit& un, int j) -> bool {
          const int nst = is_k ? K_STAGES : V_STAGES;
          uint64_t* fullb = is_k ? k_full : v_full;
          uint64_t* emptyb = is_k ? k_empty : v_empty;
          const CUtensorMap* map = is_k ? &tmK : &tmV;
          uint8_t* base = smem + (is_k ? Layout::OFF_K : Layout::OFF_V);
          const int st = static_cast<int>(kv_t % nst);
          const uint32_t ph = (kv_t / nst) & 1u;
          if (!mbar_wait(&emptyb[st], ph ^ 1u, abort_flag, p.status, SITE_PROD_KV)) return false;
          uint8_t* dst = base + st * TILE;
          mbar_arrive_expect_tx(&fullb[st], TILE);
          tma_load_4d(map, &fullb[st], dst, 0, un.h, j * BN, un.b);
          tma_load_4d(map, &fullb[st], dst + HALF, 64, un.h, j * BN, un.b);
          ++kv_t;
          return true;
        };
        for (int k = 0; k < rounds && ok; ++k) {
          const int u = snake(k, blockIdx.x, gridDim.x);
          if (u >= num_units) continue;
          const Unit un = unit_of(u, p);
          if (!load_kv(un, 0)) break;
          if (is_k || un.has_b) {
            if (!mbar_wait(&q_empty[qt], qphase ^ 1u, abort_flag, p.status, SITE_PROD_Q)) break;
            qphase ^= 1u;
            const int q0 = 2 * un.pair * BM + qt * BM;
            uint8_t* qdst = smem + Layout::OFF_Q + qt * TILE;
            mbar_arrive_expect_tx(&q_full[qt], TILE);
            tma_load_4d(&tmQ, &q_full[qt], qdst, 0, un.h, q0, un.b);
            tma_load_4d(&tmQ, &q_full[qt], qdst + HALF, 64, un.h, q0, un.b);
          }
          for (int j = 1; j < un.nkv && ok; ++j) ok = load_kv(un, j);
        }
      }
    } else if (warp == MMA_WARP) {
      // ------------------------------ MMA issuer ------------------------------
      // The whole warp walks the schedule (converged control flow: the shared-memory
      // descriptors are warp-uniform), one elected lane issues each group of MMAs together
      // with the commits that track it.
      constexpr uint32_t idesc_s = make_idesc(BM, BN, 1u, 1u, 0u, 0u);  // Q K^T, both K-major
      constexpr uint32_t idesc_o = make_idesc(BM, D, 1u, 1u, 0u, 1u);   // P (TMEM) V (MN-major)
      const uint64_t qdesc = sdesc_sw128(smem_u32(smem + Layout::OFF_Q), 16, 1024);
      uint32_t kv_t = 0;
      uint32_t qphase[2] = {0, 0};
      uint32_t pphase[2] = {0, 0};
      uint32_t ofree_phase[2] = {0, 0};
      int units_done = 0;
      bool s_a_issued = false;  // the unit's S_A(0) went out during the previous unit's tail
      bool ok = true;
      // descriptor start addresses are in 16-byte units: stepping one adds (bytes >> 4)
      auto issue_s = [&](int tile, uint64_t kdesc, uint64_t* extra0, uint64_t* extra1) {
        const uint64_t adesc = qdesc + static_cast<uint64_t>((tile * TILE) >> 4);
        if (elect_one_sync()) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = ((kk >> 2) * HALF + (kk & 3) * 32) >> 4;
            umma_f16(tmem + t_s_col(tile), adesc + off, kdesc + off, idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[tile]);
          if (extra0 != nullptr) umma_commit(extra0);
          if (extra1 != nullptr) umma_commit(extra1);
        }
        __syncwarp();
      };
      // O_t of the previous unit must have been read by its epilogue before the first PV of
      // tile t overwrites it; the S MMAs of the new unit do not touch O and go ahead of that
      auto wait_o_free = [&](int tile) -> bool {
        if (units_done == 0) return true;
        if (!mbar_wait(&o_free[tile], ofree_phase[tile], abort_flag, p.status, SITE_MMA_OFREE)) {
          return false;
        }
        ofree_phase[tile] ^= 1u;
        tc_fence_after();
        return true;
      };
      auto issue_pv = [&](int tile, uint64_t vdesc, bool first, uint64_t* done0,
                          uint64_t* done1) -> bool {
        if (first && !wait_o_free(tile)) return false;
        // P arrives in two halves (keys 0-63, 64-127): the first half of PV starts while the
        // softmax still works on the second
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (!mbar_wait(&p_full[2 * tile + h], pphase[tile], abort_flag, p.status,
                         SITE_MMA_P)) {
            return false;
          }
          tc_fence_after();
          if (elect_one_sync()) {
#pragma unroll
            for (int kk = h * BN / 32; kk < (h + 1) * BN / 32; ++kk) {
              umma_f16_tmem_a(tmem + t_o_col(tile), tmem + t_s_col(tile) + kk * 8,
                              vdesc + static_cast<uint64_t>(kk * 16 * 128 / 16), idesc_o,
                              (!first || kk > 0) ? 1u : 0u);
            }
            if (h == 1 && done0 != nullptr) umma_commit(done0);
            if (h == 1 && done1 != nullptr) umma_commit(done1);
          }
          __syncwarp();
        }
        pphase[tile] ^= 1u;
        return true;
      };
      for (int k = 0; k < rounds && ok; ++k) {
        const int u = snake(k, blockIdx.x, gridDim.x);
        if (u >= num_units) continue;
        const Unit un = unit_of(u, p);
        if (!s_a_issued) {
          if (!mbar_wait(&q_full[0], qphase[0], abort_flag, p.status, SITE_MMA_Q)) break;
          qphase[0] ^= 1u;
        }
        tc_fence_after();
        const int a_last = 2 * un.pair;  // tile A's diagonal KV tile
        uint64_t prev_vdesc = 0;
        for (int j = 0; j < un.nkv && ok; ++j, ++kv_t) {
          const int ks = static_cast<int>(kv_t % K_STAGES);
          const int vs = static_cast<int>(kv_t % V_STAGES);
          const bool pre = j == 0 && s_a_issued;  // K(0) was waited for in the tail
          if (!pre && !mbar_wait(&k_full[ks], (kv_t / K_STAGES) & 1u, abort_flag, p.status,
                                 SITE_MMA_K)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t kdesc = sdesc_sw128(smem_u32(smem + Layout::OFF_K + ks * TILE), 16, 1024);
          const uint64_t vdesc =
              sdesc_sw128(smem_u32(smem + Layout::OFF_V + vs * TILE), HALF, 1024);
          const bool a_on = j <= a_last;
          // K(j) is released by the commit after its last reader; each Q tile after its
          // tile's last S
          if (a_on && !pre) {
            issue_s(0, kdesc, un.has_b ? nullptr : &k_empty[ks],
                    j == a_last ? &q_empty[0] : nullptr);
          }
          if (un.has_b && j > 0) {
            // V(j-1) is free once PV_B(j-1) (and everything before it) completed
            if (!issue_pv(1, prev_vdesc, j - 1 == 0, &v_empty[(kv_t - 1) % V_STAGES], nullptr)) {
              ok = false;
              break;
            }
          }
          if (un.has_b) {
            if (j == 0) {
              if (!mbar_wait(&q_full[1], qphase[1], abort_flag, p.status, SITE_MMA_Q)) {
                ok = false;
                break;
              }
              qphase[1] ^= 1u;
              tc_fence_after();
            }
            issue_s(1, kdesc, &k_empty[ks], j == un.nkv - 1 ? &q_empty[1] : nullptr);
          }
          if (!mbar_wait(&v_full[vs], (kv_t / V_STAGES) & 1u, abort_flag, p.status,
                         SITE_MMA_V)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (a_on) {
            if (!issue_pv(0, vdesc, j == 0, j == a_last ? &o_done[0] : nullptr,
                          un.has_b ? nullptr : &v_empty[vs])) {
              ok = false;
              break;
            }
          }
          prev_vdesc = vdesc;
        }
        if (!ok) break;
        // Tail: the last step is tile B's alone, and its PV waits for the softmax of B's
        // diagonal tile. When the next unit's Q_A and first K tile have landed, its S_A(0)
        // goes to the tensor core now (after this unit's last PV_A: in order), so that the
        // tensor core and tile A's softmax work while B's finishes.
        s_a_issued = false;
        if (p.tail && un.has_b && k + 1 < rounds) {
          const int v = snake(k + 1, blockIdx.x, gridDim.x);
          if (v < num_units) {
            const Unit nx = unit_of(v, p);
            const int ks = static_cast<int>(kv_t % K_STAGES);
            const int ready = (mbar_test(&q_full[0], qphase[0]) &&
                               mbar_test(&k_full[ks], (kv_t / K_STAGES) & 1u)) ? 1 : 0;
            if (__shfl_sync(0xffffffffu, ready, 0)) {
              qphase[0] ^= 1u;
              tc_fence_after();
              const uint64_t kdesc =
                  sdesc_sw128(smem_u32(smem + Layout::OFF_K + ks * TILE), 16, 1024);
              issue_s(0, kdesc, nx.has_b ? nullptr : &k_empty[ks],
                      nx.pair == 0 ? &q_empty[0] : nullptr);  // S_A(0) is A's last S then
              s_a_issued = true;
            }
          }
        }
        if (un.has_b) {
          if (!issue_pv(1, prev_vdesc, un.nkv - 1 == 0, &o_done[1],
                        &v_empty[(kv_t - 1) % V_STAGES])) {
            break;
          }
        } else {
          // tile B absent: hand O_B back once the previous unit's epilogue has read it
          if (!wait_o_free(1)) break;
          if (elect_one_sync()) umma_commit(&o_done[1]);
          __syncwarp();
        }
        ++units_done;
      }
    }
  } else {
    setmaxnreg_inc<SOFTMAX_REGS>();
    // ------------- softmax, O correction and epilogue (thread = query row) -------------
    const int tile = warp >> 2;              // 0: tile A (warps 0-3), 1: tile B (warps 4-7)
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tmem + lane_base + t_s_col(tile);
    const uint32_t t_o = tmem + lane_base + t_o_col(tile);
    const float sl = p.scale_log2;
    uint32_t sphase = 0, ophase = 0;
    bool ok = true;
    for (int k = 0; k < rounds && ok; ++k) {
      const int u = snake(k, blockIdx.x, gridDim.x);
      if (u >= num_units) continue;
      const Unit un = unit_of(u, p);
      const bool active = tile == 0 || un.has_b;
      const int qt = 2 * un.pair + tile;       // this warpgroup's query tile
      float m_used = -INFINITY;                // log2-domain maximum of the exponentials
      float lsum = 0.f;
      if (active) {
        for (int j = 0; j <= qt; ++j) {
          if (!mbar_wait(&s_full[tile], sphase, abort_flag, p.status, SITE_SM_S)) {
            ok = false;
            break;
          }
          sphase ^= 1u;
          tc_fence_after();
          if (j == qt) {
            softmax_step<true>(t_s, t_o, row, lane, sl, m_used, lsum, &p_full[2 * tile]);
          } else {
            softmax_step<false>(t_s, t_o, row, lane, sl, m_used, lsum, &p_full[2 * tile]);
          }
        }
        if (!ok) break;
      }
      // ---- epilogue: O / l -> bf16 rows -> global; LSE ----
      if (!mbar_wait(&o_done[tile], ophase, abort_flag, p.status, SITE_SM_O)) break;
      ophase ^= 1u;
      tc_fence_after();
      const int qrow = qt * BM + row;
      if (active) {
        const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
        __nv_bfloat16* orow =
            p.out + ((static_cast<long long>(un.b) * p.seq + qrow) * p.heads + un.h) * D;
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_o + c, r);
          tmem_ld_wait();
          reg_fence(r);
          if (qrow < p.seq) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              pk[i] = pack_bf16x2(__uint_as_float(r[2 * i]) * inv,
                                  __uint_as_float(r[2 * i + 1]) * inv);
            }
            uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
            }
          }
        }
        if (qrow < p.seq) {
          p.lse[(static_cast<long long>(un.b) * p.heads + un.h) * p.seq + qrow] =
              (m_used + __log2f(lsum)) * 0.6931471805599453f;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[tile]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
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
  if (B > 65535 || H > 65535 || S > (1 << 24) || B * H * ((S + 2 * BM - 1) / (2 * BM)) > (1LL << 31) - 1) {
    return KTA_ERR_UNSUPPORTED;
  }
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O) ||
      (reinterpret_cast<uintptr_t>(LSE) & 3)) {
    return KTA_ERR_ALIGN;
  }
  int s = require_sm100();
  if (s != KTA_OK) return s;
  // [B, S, H, D] as a 4-D map: d innermost, then h, s, b (rows past S of a batch entry
  // read as zeros)
  const uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(H),
                            static_cast<uint64_t>(S), static_cast<uint64_t>(B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(H * D) * 2,
                               static_cast<uint64_t>(S * H * D) * 2};
  const uint32_t box[4] = {64, 1, 128, 1};
  CUtensorMap tq, tk, tv;
  const void* ptrs[3] = {Q, K, V};
  CUtensorMap* maps[3] = {&tq, &tk, &tv};
  for (int i = 0; i < 3; ++i) {
    s = encode_tmap(maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, ptrs[i], dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  Params prm;
  prm.out = static_cast<__nv_bfloat16*>(O);
  prm.lse = static_cast<float*>(LSE);
  prm.batch = static_cast<int>(B);
  prm.heads = static_cast<int>(H);
  prm.seq = static_cast<int>(S);
  prm.q_tiles = static_cast<int>((S + BM - 1) / BM);
  prm.pairs = (prm.q_tiles + 1) / 2;
  prm.scale_log2 = scale * 1.4426950408889634f;
  // KTA_ATTN_TAIL=0 switches the tail overlap off (comparison runs)
  prm.tail = 1;
  if (const char* e = std::getenv("KTA_ATTN_TAIL")) prm.tail = std::atoi(e) != 0;
  // cost-major unit order when all heads' K and V (B H S D 4 bytes) take at most 96 MB of the
  // 126 MB L2; KTA_ATTN_ORDER=head|cost overrides (comparison runs)
  prm.cost_major = B * H * S * D * 4 <= (int64_t{96} << 20) ? 1 : 0;
  if (const char* e = std::getenv("KTA_ATTN_ORDER")) prm.cost_major = e[0] == 'c' ? 1 : 0;
  prm.status = device_status_ptr();
  s = set_kernel_smem(reinterpret_cast<const void*>(attn_fwd_kernel), Layout::ALLOC);
  if (s != KTA_OK) return s;
  const long long units = B * H * static_cast<long long>(prm.pairs);
  const int grid = static_cast<int>(std::max(1LL, std::min<long long>(current_sm_count(), units)));
  return launch_ex(attn_fwd_kernel, dim3(grid), dim3(NUM_THREADS), Layout::ALLOC, stream, 1, tq,
                   tk, tv, prm);
}

}  // namespace attn
}  // namespace kta

extern "C" int kta_attn_fwd_causal_bf16(const void* Q, const void* K, const void* V, void* O,
                                        void* LSE, int64_t B, int64_t H, int64_t S, int64_t D,
                                        float scale, void* stream) {
  return kta::attn::launch(Q, K, V, O, LSE, B, H, S, D, scale, static_cast<cudaStream_t>(stream));
}
