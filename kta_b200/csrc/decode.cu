// GQA decode attention, sm_100a: one query token per sequence over a packed, per-sequence
// contiguous bf16 KV cache of variable lengths.
//
// It replaces KTA's TileLang flash-decoding pair decode_partial / decode_combine
// (perfmodel/testset/gen.py:493-590): split the KV sequence, compute per split the
// normalised partial output and its log-sum-exp in log2 units (gen.py:553), then combine the
// splits with exp2 weights (gen.py:579-588). B200-first design:
//
//   * the work is the list of 128-token tiles of every (sequence, KV head) pair; a
//     persistent grid of one CTA per SM takes one contiguous range of that list each
//     (stream-K style), so variable lengths balance to within a tile and a CTA touches only
//     a few pairs ("segments"); a pair split between CTAs is finished by the CTA that
//     completes it last (arrival counter, partials in the caller's workspace);
//   * a producer warp streams K, V (3-D TMA maps over [T, Hkv, D], 128-byte swizzle) and the
//     group's query rows into a 3-stage mbarrier ring: the HBM reads stay in flight while
//     eight compute warps work;
//   * compute warps take 16 tokens of each tile in transposed form on mma.sync m16n8k16:
//     S^T = K Q^T (tokens on M), exp2 online softmax per query head, P^T re-laid as the B
//     operand with movmatrix, O^T += V^T P^T; tensor time is far below the KV stream;
//   * at the end of a segment the compute warps drop their (m, l, O) into shared memory and
//     continue at once: a merger warp folds the eight states and writes the output or the
//     partial, so merges never stall the KV stream; the CTA's last segment, which ends the
//     stream, the eight compute warps fold themselves (and combine the pair when this CTA
//     is its last contributor), 256 threads instead of one warp on the kernel's tail;
//   * every mbarrier wait is bounded; out-of-range lengths/offsets are rejected on the
//     device (status KTA_ERR_DEVICE_BOUNDS) and that sequence's output is zero-filled.
#include <algorithm>
#include <cmath>
#include <mutex>

#include "kta_common.cuh"
#include "kta_host.h"

namespace kta {
namespace decode {

constexpr int D = 128;
constexpr int TILE = 128;                     // tokens per TMA tile
constexpr int COMPUTE_WARPS = TILE / 16;      // 16 tokens per compute warp
constexpr int PRODUCER_WARP = COMPUTE_WARPS;
constexpr int MERGER_WARP = COMPUTE_WARPS + 1;
constexpr int NUM_THREADS = 32 * (COMPUTE_WARPS + 2);
constexpr int MAX_BATCH = 2048;
constexpr int MAX_GROUP = 16;
constexpr int MAX_GRID = 256;                 // workspace is sized for this many CTAs
constexpr int HALF_BYTES = TILE * 64 * 2;     // one 64-wide half of a K or V tile
constexpr int TILE_BYTES = 2 * HALF_BYTES;    // a full [TILE, 128] bf16 tile
constexpr int Q_HALF_BYTES = 2048;            // [<=16 heads, 64] bf16, 128-byte swizzle
constexpr int STAGE_BYTES = 2 * TILE_BYTES + 2 * Q_HALF_BYTES;  // K, V and the segment's Q

enum : unsigned int {
  SITE_PROD_EMPTY = 0x301,
  SITE_CONS_FULL = 0x302,
  SITE_CONS_MFREE = 0x303,
  SITE_MERGE_FULL = 0x304,
  SITE_CONS_GROUP = 0x305,
};

struct Params {
  const int32_t* seqlens;      // [B]
  const int64_t* offsets;      // [B]
  __nv_bfloat16* out;          // [B, Hq, D]
  unsigned int* counters;      // [B * Hkv] arrivals per split pair
  float* part_lse;             // [2 * MAX_GRID, G] log2-unit LSE of a partial segment
  float* part_o;               // [2 * MAX_GRID, G, D] normalised partial output
  int batch, hq, hkv, group, max_seqlen;
  long long cache_tokens;
  float scale_log2;            // softmax scale * log2(e)
  unsigned int* status;
};

// Shared-memory layout (runtime: the merge area scales with G, the tables with B).
struct Smem {
  int off_merge_o, off_merge_ml, off_tiles, off_prefix, off_bar, off_misc, total;
  __host__ __device__ Smem(int stages, int G, int B) {
    off_merge_o = stages * STAGE_BYTES;                       // [warps][G][D] fp32
    off_merge_ml = off_merge_o + COMPUTE_WARPS * G * D * 4;   // [warps][G][2] fp32
    off_tiles = off_merge_ml + COMPUTE_WARPS * G * 2 * 4;     // [B] tiles per pair, -1 bad
    off_prefix = off_tiles + B * 4;                           // [B + 1] tiles before b
    off_bar = ((off_prefix + (B + 1) * 4 + 7) / 8) * 8;
    off_misc = off_bar + (2 * stages + 3) * 8;
    total = off_misc + 32;
  }
};

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32"
      " {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Address of the 16-byte chunk `chunk` (0..7) of row `row` in a 128-byte-swizzled block.
__device__ __forceinline__ uint32_t swz(uint32_t base, int row, int chunk) {
  return base + static_cast<uint32_t>(row) * 128u +
         (static_cast<uint32_t>(chunk ^ (row & 7)) << 4);
}

// The tile list: pairs (b, kvh) in b-major order, tiles(b) tiles each. CTA c owns
// [start(c), start(c + 1)) with start(c) = floor(c * total / grid).
struct Work {
  const int* tiles;   // [B]
  const int* prefix;  // [B + 1] tiles of all pairs of sequences before b
  int batch, hkv, grid;
  long long total;

  __device__ __forceinline__ long long start(int c) const { return total * c / grid; }
  // CTA c has at least one tile (with fewer tiles than CTAs, some ranges are empty)
  __device__ __forceinline__ bool busy(int c) const { return start(c + 1) > start(c); }
  // CTA owning global tile t
  __device__ __forceinline__ int owner(long long t) const {
    return static_cast<int>(((t + 1) * grid - 1) / total);
  }
};

struct Segment {
  int b, kvh;            // the pair
  int i0, i1;            // tiles [i0, i1) of the pair
  int ntiles;            // tiles of the pair
  long long pair_start;  // global index of the pair's first tile
  long long next;        // global index after this segment
};

__device__ __forceinline__ Segment segment_at(const Work& w, long long t, long long end) {
  int lo = 0, hi = w.batch - 1;
  while (lo < hi) {  // sequence b with prefix[b] <= t < prefix[b + 1]
    const int mid = (lo + hi) >> 1;
    if (w.prefix[mid + 1] > t) {
      hi = mid;
    } else {
      lo = mid + 1;
    }
  }
  Segment s;
  s.b = lo;
  s.ntiles = w.tiles[lo];
  const long long rel = t - w.prefix[lo];
  s.kvh = static_cast<int>(rel / s.ntiles);
  s.i0 = static_cast<int>(rel - static_cast<long long>(s.kvh) * s.ntiles);
  s.pair_start = t - s.i0;
  const long long pair_end = s.pair_start + s.ntiles;
  s.next = pair_end < end ? pair_end : end;
  s.i1 = static_cast<int>(s.next - s.pair_start);
  return s;
}

// The threads that fold a segment's eight warp states: the merger warp (segments that end
// while the CTA still streams) or the eight compute warps (the CTA's last segment, when they
// have nothing else to do). sync() orders the group's shared- and global-memory writes before
// every member's later accesses; the compute warps' version waits on an mbarrier with the
// library's bounded wait, so if one warp gave up earlier the others stop at the wait's limit
// (and record it) instead of waiting for good.
struct WarpGroup {
  static constexpr int THREADS = 32;
  static constexpr int COMBINE_NC = 4;  // pieces whose loads go out together
  static constexpr int COMBINE_U = 8;   // output elements per thread and pass
  int ti;
  __device__ __forceinline__ bool sync() {
    __syncwarp();
    return true;
  }
};
struct ComputeGroup {
  static constexpr int THREADS = COMPUTE_WARPS * 32;
  static constexpr int COMBINE_NC = 8;
  static constexpr int COMBINE_U = 2;
  int ti;
  uint64_t* bar;  // count COMPUTE_WARPS: one arrival per warp
  uint32_t phase;
  volatile int* abort;
  unsigned int* status;
  __device__ __forceinline__ bool sync() {
    __syncwarp();
    if ((ti & 31) == 0) mbar_arrive(bar);
    const bool ok = mbar_wait(bar, phase, abort, status, SITE_CONS_GROUP);
    phase ^= 1u;
    return ok;
  }
};

// Folds segment sg's eight warp states (merge_o [warps][G][D], merge_ml [warps][G][2] = m, l)
// into the output of a whole pair, or into partial slot `slot` (normalised O and the LSE in
// log2 units) of a split one. Thread g < G turns head g's states into one normalised weight
// per warp, written over that warp's m, and the head's LSE, written over warp 0's l (only
// thread g touches head g's entries); every element is then a weighted sum of eight values.
template <typename Group>
__device__ bool fold_segment(Group& grp, const Params& p, const Segment& sg, bool partial,
                             int slot, int G, float* merge_o, float* merge_ml) {
  for (int g = grp.ti; g < G; g += Group::THREADS) {
    float M = -INFINITY;
#pragma unroll
    for (int wi = 0; wi < COMPUTE_WARPS; ++wi) M = fmaxf(M, merge_ml[(wi * G + g) * 2]);
    float fw[COMPUTE_WARPS];
    float Lsum = 0.f;
#pragma unroll
    for (int wi = 0; wi < COMPUTE_WARPS; ++wi) {
      const float mw = merge_ml[(wi * G + g) * 2];
      fw[wi] = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      Lsum += merge_ml[(wi * G + g) * 2 + 1] * fw[wi];
    }
    const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
#pragma unroll
    for (int wi = 0; wi < COMPUTE_WARPS; ++wi) merge_ml[(wi * G + g) * 2] = fw[wi] * inv;
    merge_ml[g * 2 + 1] = Lsum > 0.f ? M + __log2f(Lsum) : -INFINITY;
  }
  if (!grp.sync()) return false;
  for (int idx = grp.ti; idx < G * D; idx += Group::THREADS) {
    const int g = idx / D, d = idx - g * D;
    float val = 0.f;
#pragma unroll
    for (int wi = 0; wi < COMPUTE_WARPS; ++wi) {
      val += merge_o[(wi * G + g) * D + d] * merge_ml[(wi * G + g) * 2];
    }
    if (!partial) {
      p.out[(static_cast<long long>(sg.b) * p.hq + sg.kvh * G + g) * D + d] =
          __float2bfloat16_rn(val);
    } else {
      p.part_o[(static_cast<long long>(slot) * G + g) * D + d] = val;
      if (d == 0) p.part_lse[slot * G + g] = merge_ml[g * 2 + 1];
    }
  }
  return true;
}

// After a split segment's partial stores: counts this CTA's arrival on the pair, and the last
// of the pair's CTAs combines every piece (decode_combine): Group::COMBINE_NC contributors at
// a time with all their loads issued at once, a running maximum rescaling the sums between
// groups, Group::COMBINE_U output elements per thread and pass (the warp: 4 pieces x 8
// elements, two passes for G = 4; the compute warps: 8 pieces x 2 elements, one pass), so a
// pair spread over up to eight CTAs costs one or two L2 round trips per pass. `flag` is a
// shared int of this group.
template <typename Group>
__device__ void arrive_and_combine(Group& grp, const Params& p, const Work& w, const Segment& sg,
                                   int G, volatile int* flag) {
  const int pair = sg.b * p.hkv + sg.kvh;
  const long long pair_end = sg.pair_start + sg.ntiles;
  const int c_first = w.owner(sg.pair_start);
  const int c_last = w.owner(pair_end - 1);
  // every member's partial stores precede thread 0's fence, which is cumulative
  if (!grp.sync()) return;
  if (grp.ti == 0) {
    int n = 0;  // CTAs holding a piece of this pair
    for (int c = c_first; c <= c_last; ++c) n += w.busy(c) ? 1 : 0;
    __threadfence();
    const unsigned int prev = atomicAdd(p.counters + pair, 1u);
    const int last = (prev == static_cast<unsigned int>(n - 1)) ? 1 : 0;
    if (last) __threadfence();
    *flag = last;
  }
  if (!grp.sync()) return;
  if (*flag == 0) return;
  constexpr int NC = Group::COMBINE_NC, U = Group::COMBINE_U;
  const int ncon = c_last - c_first + 1;
  for (int base = 0; base < G * D; base += Group::THREADS * U) {
    int gi[U], di[U];
    bool vi[U];
    float mx[U], wsum[U], acc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = base + u * Group::THREADS + grp.ti;
      vi[u] = e < G * D;
      gi[u] = vi[u] ? e / D : 0;
      di[u] = vi[u] ? e - gi[u] * D : 0;
      mx[u] = -INFINITY;
      wsum[u] = 0.f;
      acc[u] = 0.f;
    }
    for (int j0 = 0; j0 < ncon; j0 += NC) {
      float lse[NC][U], ov[NC][U];
#pragma unroll
      for (int j = 0; j < NC; ++j) {
        const int c = c_first + j0 + j;
        const bool on = j0 + j < ncon && w.busy(c);
        const int sl = on ? 2 * c + (w.start(c) >= sg.pair_start ? 0 : 1) : 0;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const bool ld = on && vi[u];
          lse[j][u] = ld ? __ldcg(p.part_lse + sl * G + gi[u]) : -INFINITY;
          ov[j][u] = ld ? __ldcg(p.part_o + (static_cast<long long>(sl) * G + gi[u]) * D + di[u])
                        : 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float cmx = -INFINITY;
#pragma unroll
        for (int j = 0; j < NC; ++j) cmx = fmaxf(cmx, lse[j][u]);
        const float nmx = fmaxf(mx[u], cmx);
        if (nmx != -INFINITY) {
          const float sc = (mx[u] == -INFINITY) ? 0.f : exp2f(mx[u] - nmx);
          wsum[u] *= sc;
          acc[u] *= sc;
#pragma unroll
          for (int j = 0; j < NC; ++j) {
            const float wt = (lse[j][u] == -INFINITY) ? 0.f : exp2f(lse[j][u] - nmx);
            wsum[u] += wt;
            acc[u] += wt * ov[j][u];
          }
          mx[u] = nmx;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (vi[u]) {
        p.out[(static_cast<long long>(sg.b) * p.hq + sg.kvh * G + gi[u]) * D + di[u]] =
            __float2bfloat16_rn(wsum[u] > 0.f ? acc[u] / wsum[u] : 0.f);
      }
    }
  }
  if (grp.ti == 0) p.counters[pair] = 0u;  // ready for the next call
}

// NT = number of 8-wide query-head tiles (1: G <= 8, 2: G <= 16).
template <int STAGES, int NT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const __grid_constant__ CUtensorMap tmQ, const Params p) {
  const Smem L(STAGES, p.group, p.batch);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  float* merge_o = reinterpret_cast<float*>(smem + L.off_merge_o);
  float* merge_ml = reinterpret_cast<float*>(smem + L.off_merge_ml);
  int* s_tiles = reinterpret_cast<int*>(smem + L.off_tiles);
  int* prefix = reinterpret_cast<int*>(smem + L.off_prefix);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.off_bar);
  uint64_t* empty = full + STAGES;
  uint64_t* mfull = empty + STAGES;   // compute warps -> merger: states are in smem
  uint64_t* mfree = mfull + 1;        // merger -> compute warps: merge area is free
  uint64_t* csync = mfree + 1;        // the compute warps among themselves (last segment)
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.off_misc);
  volatile int* merger_flag = abort_flag + 2;   // "this CTA combines the pair" for the merger
  volatile int* compute_flag = abort_flag + 3;  // ... and for the compute warps

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  const int B = p.batch;
  const int G = p.group;

  pdl_launch_dependents();
  pdl_wait();  // the previous grid's writes (this launch's inputs) are visible from here on
  // ---- lengths, validation and the tile prefix (every CTA computes the same table) ----
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int len = p.seqlens[b];
    const long long off = p.offsets[b];
    const bool bad = len < 0 || len > p.max_seqlen || off < 0 ||
                     off + static_cast<long long>(len) > p.cache_tokens;
    if (bad && blockIdx.x == 0) record_status(p.status, KTA_ERR_DEVICE_BOUNDS, 0x310);
    s_tiles[b] = bad ? -1 : (len + TILE - 1) / TILE;  // -1: rejected, 0: empty
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], COMPUTE_WARPS);
    }
    mbar_init(mfull, COMPUTE_WARPS);
    mbar_init(mfree, 1);
    mbar_init(csync, COMPUTE_WARPS);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == 0) {
    // warp-parallel exclusive scan of tiles x Hkv per sequence
    const int per = (B + 31) / 32;
    const int b0 = lane * per;
    int local = 0;
    for (int b = b0; b < min(B, b0 + per); ++b) local += max(s_tiles[b], 0) * p.hkv;
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - local;
    for (int b = b0; b < min(B, b0 + per); ++b) {
      prefix[b] = run;
      run += max(s_tiles[b], 0) * p.hkv;
    }
    if (lane == 31) prefix[B] = incl;
  }
  __syncthreads();

  Work w;
  w.tiles = s_tiles;
  w.prefix = prefix;
  w.batch = B;
  w.hkv = p.hkv;
  w.grid = gridDim.x;
  w.total = prefix[B];
  const long long my_begin = w.total > 0 ? w.start(blockIdx.x) : 0;
  const long long my_end = w.total > 0 ? w.start(blockIdx.x + 1) : 0;

  // Rejected or empty sequences: zero output (CTA 0 only).
  if (blockIdx.x == 0) {
    for (int b = 0; b < B; ++b) {
      if (s_tiles[b] <= 0) {
        for (int i = threadIdx.x; i < p.hq * D; i += blockDim.x) {
          p.out[static_cast<long long>(b) * p.hq * D + i] = __float2bfloat16_rn(0.f);
        }
      }
    }
  }

  if (warp == PRODUCER_WARP) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint32_t q_bytes = 2u * static_cast<uint32_t>(G) * 128u;
      for (long long t = my_begin; t < my_end && ok;) {
        const Segment sg = segment_at(w, t, my_end);
        const long long base = p.offsets[sg.b];
        const int qrow = sg.b * p.hq + sg.kvh * G;
        for (int i = sg.i0; i < sg.i1; ++i) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status, SITE_PROD_EMPTY)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + stage * STAGE_BYTES;
          const int tok = static_cast<int>(base + static_cast<long long>(i) * TILE);
          const bool first = i == sg.i0;
          mbar_arrive_expect_tx(&full[stage], 2 * TILE_BYTES + (first ? q_bytes : 0u));
          tma_load_3d(&tmK, &full[stage], st, 0, sg.kvh, tok);
          tma_load_3d(&tmK, &full[stage], st + HALF_BYTES, 64, sg.kvh, tok);
          tma_load_3d(&tmV, &full[stage], st + TILE_BYTES, 0, sg.kvh, tok);
          tma_load_3d(&tmV, &full[stage], st + TILE_BYTES + HALF_BYTES, 64, sg.kvh, tok);
          if (first) {  // the group's query rows, once per segment
            tma_load_2d(&tmQ, &full[stage], st + 2 * TILE_BYTES, 0, qrow);
            tma_load_2d(&tmQ, &full[stage], st + 2 * TILE_BYTES + Q_HALF_BYTES, 64, qrow);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        t = sg.next;
      }
    }
    __syncwarp();
  } else if (warp == MERGER_WARP) {
    // ------------------------------ merger ------------------------------
    // Segments that end while the CTA still streams; the CTA's last segment is folded by the
    // compute warps themselves, which are idle by then.
    WarpGroup grp{lane};
    int seg = 0;
    for (long long t = my_begin; t < my_end; ++seg) {
      const Segment sg = segment_at(w, t, my_end);
      if (sg.next >= my_end) break;
      if (!mbar_wait(mfull, static_cast<uint32_t>(seg & 1), abort_flag, p.status,
                     SITE_MERGE_FULL)) {
        break;
      }
      const bool partial = !(sg.i0 == 0 && sg.i1 == sg.ntiles);
      // Slot of a partial segment: the CTA's first segment uses 2c, its last 2c + 1.
      const int slot = 2 * static_cast<int>(blockIdx.x) + (t == my_begin ? 0 : 1);
      fold_segment(grp, p, sg, partial, slot, G, merge_o, merge_ml);
      __syncwarp();
      if (lane == 0) mbar_arrive(mfree);  // the merge area may be overwritten
      if (partial) arrive_and_combine(grp, p, w, sg, G, merger_flag);
      t = sg.next;
    }
    __syncwarp();
  } else {
    // ------------------------------ compute warps ------------------------------
    // Transposed form: tokens on the MMA's M (16 per warp), query heads on N.
    //   S^T[tok, h] = K[tok, :] . Q[h, :]          (A = K tile, B = Q)
    //   O^T[d, h]  += V^T[d, tok] . P^T[tok, h]    (A = V tile transposed, B = P^T)
    const int r0 = warp * 16;               // this warp's token rows in a tile
    const int tq = lane >> 2;               // C fragment row (token or d) of c0, c1
    const int hc = (lane & 3) * 2;          // C fragment column pair (query heads)
    int stage = 0;
    uint32_t phase = 0;
    int seg = 0;
    for (long long t = my_begin; t < my_end; ++seg) {
      const Segment sg = segment_at(w, t, my_end);
      const int len = p.seqlens[sg.b];
      uint32_t qb[NT][8][2];
      float o[8][NT][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) o[i][nt][0] = o[i][nt][1] = o[i][nt][2] = o[i][nt][3] = 0.f;
      }
      float m[NT][2], l[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        m[nt][0] = m[nt][1] = -INFINITY;
        l[nt][0] = l[nt][1] = 0.f;
      }
      bool ok = true;
      for (int i = sg.i0; i < sg.i1; ++i) {
        if (!mbar_wait(&full[stage], phase, abort_flag, p.status, SITE_CONS_FULL)) {
          ok = false;
          break;
        }
        const uint32_t kbase = smem_u32(smem + stage * STAGE_BYTES);
        const uint32_t vbase = kbase + TILE_BYTES;
        if (i == sg.i0) {
          // Q B-fragments: b0 = Q[h = nt*8 + lane/4][d = 16kk + hc], b1 = d + 8.
          const uint32_t qbase = kbase + 2 * TILE_BYTES;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int h = nt * 8 + tq;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint32_t hb = qbase + (kk >> 2) * Q_HALF_BYTES;
              const int c0 = (kk & 3) * 2;
              qb[nt][kk][0] = h < G ? lds_u32(swz(hb, h, c0) + (lane & 3) * 4) : 0u;
              qb[nt][kk][1] = h < G ? lds_u32(swz(hb, h, c0 + 1) + (lane & 3) * 4) : 0u;
            }
          }
        }
        const int valid = len - i * TILE - r0;  // tokens of this warp's slice in the sequence
        if (valid > 0) {
          // ---- S^T = K Q^T over 16 tokens ----
          float sacc[NT][4];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
          const int arow = r0 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            uint32_t a[4];
            ldmatrix_x4(swz(kbase + (kk >> 2) * HALF_BYTES, arow, (kk & 3) * 2 + (lane >> 4)), a);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma_bf16_16816(sacc[nt], a, qb[nt][kk][0], qb[nt][kk][1]);
          }
          // ---- online softmax per query head (column), exp2 form ----
          const bool in_lo = tq < valid, in_hi = tq + 8 < valid;
          bool rescale = false;
          float cf[NT][2];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float v0 = in_lo ? sacc[nt][e] * p.scale_log2 : -INFINITY;
              const float v1 = in_hi ? sacc[nt][2 + e] * p.scale_log2 : -INFINITY;
              float mx = fmaxf(v0, v1);
              mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
              mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
              mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
              const float mn = fmaxf(m[nt][e], mx);
              const float c = (mn == -INFINITY) ? 1.f : exp2f(m[nt][e] - mn);
              const float p0 = (mn == -INFINITY) ? 0.f : exp2f(v0 - mn);
              const float p1 = (mn == -INFINITY) ? 0.f : exp2f(v1 - mn);
              float sm = p0 + p1;
              sm += __shfl_xor_sync(0xffffffffu, sm, 4);
              sm += __shfl_xor_sync(0xffffffffu, sm, 8);
              sm += __shfl_xor_sync(0xffffffffu, sm, 16);
              l[nt][e] = l[nt][e] * c + sm;
              m[nt][e] = mn;
              cf[nt][e] = c;
              rescale |= (c != 1.f);
              sacc[nt][e] = p0;
              sacc[nt][2 + e] = p1;
            }
          }
          if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
            for (int d8 = 0; d8 < 8; ++d8) {
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                o[d8][nt][0] *= cf[nt][0];
                o[d8][nt][1] *= cf[nt][1];
                o[d8][nt][2] *= cf[nt][0];
                o[d8][nt][3] *= cf[nt][1];
              }
            }
          }
          // ---- P^T as the B operand: transpose the two 8x8 bf16 blocks in registers ----
          uint32_t pb[NT][2];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            pb[nt][0] = movmatrix_trans(pack_bf16x2(sacc[nt][0], sacc[nt][1]));
            pb[nt][1] = movmatrix_trans(pack_bf16x2(sacc[nt][2], sacc[nt][3]));
          }
          // ---- O^T += V^T P^T: 8 tiles of 16 d ----
          const int vrow = r0 + (lane & 7) + (lane >> 4) * 8;
#pragma unroll
          for (int d8 = 0; d8 < 8; ++d8) {
            uint32_t a[4];
            ldmatrix_x4_trans(
                swz(vbase + (d8 >> 2) * HALF_BYTES, vrow, (d8 & 3) * 2 + ((lane >> 3) & 1)), a);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma_bf16_16816(o[d8][nt], a, pb[nt][0], pb[nt][1]);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;  // bounded wait gave up: the merger's own bounded wait ends it too
      // ---- hand this warp's state to the merger ----
      if (seg > 0 && !mbar_wait(mfree, static_cast<uint32_t>((seg - 1) & 1), abort_flag,
                                p.status, SITE_CONS_MFREE)) {
        break;
      }
      {
        float* mo = merge_o + warp * G * D;
        float* ml = merge_ml + warp * G * 2;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int h = nt * 8 + hc + e;
            if (h < G) {
#pragma unroll
              for (int d8 = 0; d8 < 8; ++d8) {
                mo[h * D + d8 * 16 + tq] = o[d8][nt][e];
                mo[h * D + d8 * 16 + tq + 8] = o[d8][nt][2 + e];
              }
              if (tq == 0) {
                ml[h * 2] = m[nt][e];
                ml[h * 2 + 1] = l[nt][e];
              }
            }
          }
        }
      }
      if (sg.next >= my_end) {
        // The CTA's last segment: the eight compute warps fold it (and combine the pair if
        // this CTA is its last contributor) instead of handing it to the merger warp.
        ComputeGroup grp{static_cast<int>(threadIdx.x), csync, 0u, abort_flag, p.status};
        if (grp.sync()) {  // every warp's state is in shared memory
          const bool partial = !(sg.i0 == 0 && sg.i1 == sg.ntiles);
          const int slot = 2 * static_cast<int>(blockIdx.x) + (t == my_begin ? 0 : 1);
          if (fold_segment(grp, p, sg, partial, slot, G, merge_o, merge_ml) && partial) {
            arrive_and_combine(grp, p, w, sg, G, compute_flag);
          }
        }
        break;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(mfull);
      t = sg.next;
    }
  }
  __syncthreads();
}

size_t workspace_bytes(long long B, long long hq, long long hkv) {
  const long long group = hq / hkv;
  const size_t counters = ((static_cast<size_t>(B * hkv) * 4 + 255) / 256) * 256;
  const size_t lse = ((static_cast<size_t>(2 * MAX_GRID * group) * 4 + 255) / 256) * 256;
  const size_t o = static_cast<size_t>(2 * MAX_GRID * group * D) * 4;
  return counters + lse + o;
}

int launch(const void* Q, const void* Kc, const void* Vc, const void* seqlens,
           const void* kv_offsets, void* O, int64_t B, int64_t Hq, int64_t Hkv, int64_t Dm,
           int64_t cache_tokens, int64_t max_seqlen, float scale, void* workspace,
           size_t ws_bytes, cudaStream_t stream) {
  if (!Q || !Kc || !Vc || !seqlens || !kv_offsets || !O) return KTA_ERR_INVALID_ARG;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || cache_tokens <= 0 || max_seqlen <= 0) {
    return KTA_ERR_INVALID_ARG;
  }
  if (!(scale > 0.f) || !std::isfinite(scale)) return KTA_ERR_INVALID_ARG;
  if (Dm != D || Hq % Hkv != 0 || Hq / Hkv > MAX_GROUP || B > MAX_BATCH) {
    return KTA_ERR_UNSUPPORTED;
  }
  // tile indices stay in int32 with room for a tile of overhang
  if (cache_tokens > (1LL << 31) - 1 - TILE || max_seqlen > (1LL << 30) ||
      B * Hkv * ((max_seqlen + TILE - 1) / TILE) > (1LL << 31) - 1) {
    return KTA_ERR_UNSUPPORTED;
  }
  if (!aligned16(Q) || !aligned16(Kc) || !aligned16(Vc) || !aligned16(O)) return KTA_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(seqlens) & 3) || (reinterpret_cast<uintptr_t>(kv_offsets) & 7)) {
    return KTA_ERR_ALIGN;
  }
  const size_t need = workspace_bytes(B, Hq, Hkv);
  if (workspace == nullptr || ws_bytes < need || !aligned16(workspace)) return KTA_ERR_WORKSPACE;
  int s = require_sm100();
  if (s != KTA_OK) return s;

  CUtensorMap tk, tv, tq;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(Hkv),
                              static_cast<uint64_t>(cache_tokens)};
    const uint64_t strides[2] = {static_cast<uint64_t>(D) * 2,
                                 static_cast<uint64_t>(Hkv * D) * 2};
    const uint32_t box[3] = {64, 1, TILE};
    s = encode_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, Kc, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
    s = encode_tmap(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, Vc, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }
  const long long group = Hq / Hkv;
  {
    const uint64_t qd[2] = {static_cast<uint64_t>(D), static_cast<uint64_t>(B * Hq)};
    const uint64_t qs[1] = {static_cast<uint64_t>(D) * 2};
    const uint32_t qbox[2] = {64, static_cast<uint32_t>(group)};
    s = encode_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Q, qd, qs, qbox,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KTA_OK) return s;
  }

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t counters_bytes = ((static_cast<size_t>(B * Hkv) * 4 + 255) / 256) * 256;
  const size_t lse_bytes = ((static_cast<size_t>(2 * MAX_GRID * group) * 4 + 255) / 256) * 256;
  Params prm;
  prm.seqlens = static_cast<const int32_t*>(seqlens);
  prm.offsets = static_cast<const int64_t*>(kv_offsets);
  prm.out = static_cast<__nv_bfloat16*>(O);
  prm.counters = reinterpret_cast<unsigned int*>(ws);
  prm.part_lse = reinterpret_cast<float*>(ws + counters_bytes);
  prm.part_o = reinterpret_cast<float*>(ws + counters_bytes + lse_bytes);
  prm.batch = static_cast<int>(B);
  prm.hq = static_cast<int>(Hq);
  prm.hkv = static_cast<int>(Hkv);
  prm.group = static_cast<int>(group);
  prm.max_seqlen = static_cast<int>(max_seqlen);
  prm.cache_tokens = cache_tokens;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.status = device_status_ptr();

  const int smem3 = Smem(3, prm.group, prm.batch).total + 1024;
  const bool three = smem3 <= 232448;
  const int smem_bytes = three ? smem3 : Smem(2, prm.group, prm.batch).total + 1024;
  const int grid = std::max(1, std::min(current_sm_count(), MAX_GRID));
  auto go = [&](auto kernel) -> int {
    int st = set_kernel_smem(reinterpret_cast<const void*>(kernel), 232448);
    if (st != KTA_OK) return st;
    return launch_ex(kernel, dim3(grid), dim3(NUM_THREADS), smem_bytes, stream, 1, tk, tv, tq,
                     prm);
  };
  if (group <= 8) {
    s = three ? go(decode_kernel<3, 1>) : go(decode_kernel<2, 1>);
  } else {
    s = three ? go(decode_kernel<3, 2>) : go(decode_kernel<2, 2>);
  }
  if (s != KTA_OK) return s;
  return launch_status();
}

// ---------------------------------------------------------------------------------------
// Allocation-free variant: the workspace is a fixed array in device memory that belongs to
// the library, so a caller that may not allocate device memory passes only its own inputs
// and outputs. Every GPU that loads the library holds this array until the process exits.
// ---------------------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocDevice {
  std::once_flag once;
  void* ptr = nullptr;  // device address of g_noalloc_scratch on this device
  int status = KTA_OK;
};
NoAllocDevice g_noalloc_devices[64];

// Device address of the scratch array on the current device. The host-side name of the
// array is only a stand-in: the address comes from cudaGetSymbolAddress, resolved once per
// device with that device current (the first allocation-free call on a device does it).
void* noalloc_scratch(int* status) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    (void)cudaGetLastError();
    *status = KTA_ERR_NO_DEVICE;
    return nullptr;
  }
  NoAllocDevice& d = g_noalloc_devices[dev];
  std::call_once(d.once, [&d]() {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      d.status = KTA_ERR_CUDA;
    } else {
      d.ptr = p;
    }
  });
  *status = d.status;
  return d.ptr;
}

int launch_noalloc(const void* Q, const void* Kc, const void* Vc, const void* seqlens,
                   const void* kv_offsets, void* O, int64_t B, int64_t Hq, int64_t Hkv,
                   int64_t Dm, int64_t cache_tokens, int64_t max_seqlen, float scale,
                   cudaStream_t stream) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0) return KTA_ERR_INVALID_ARG;
  if (Hq / Hkv > MAX_GROUP || B > MAX_BATCH) return KTA_ERR_UNSUPPORTED;
  // The partials and arrival counters this call needs must fit in the fixed array.
  if (workspace_bytes(B, Hq, Hkv) > kNoAllocScratchBytes) return KTA_ERR_UNSUPPORTED;
  int s = KTA_OK;
  void* scratch = noalloc_scratch(&s);
  if (scratch == nullptr) return s;
  // The array keeps whatever the previous call left; the arrival counters must start at
  // zero, so clear them on the caller's stream ahead of the kernel.
  const size_t counters_bytes = ((static_cast<size_t>(B * Hkv) * 4 + 255) / 256) * 256;
  if (cudaMemsetAsync(scratch, 0, counters_bytes, stream) != cudaSuccess) {
    (void)cudaGetLastError();
    return KTA_ERR_CUDA;
  }
  return launch(Q, Kc, Vc, seqlens, kv_offsets, O, B, Hq, Hkv, Dm, cache_tokens, max_seqlen,
                scale, scratch, kNoAllocScratchBytes, stream);
}

}  // namespace decode
}  // namespace kta

extern "C" {

size_t kta_decode_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                                  int64_t max_seqlen) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || D != kta::decode::D || Hq % Hkv != 0 || max_seqlen <= 0) {
    return 0;
  }
  return kta::decode::workspace_bytes(B, Hq, Hkv);
}

int kta_decode_gqa_bf16(const void* Q, const void* Kc, const void* Vc, const void* seqlens,
                        const void* kv_offsets, void* O, int64_t B, int64_t Hq, int64_t Hkv,
                        int64_t D, int64_t cache_tokens, int64_t max_seqlen, float scale,
                        void* workspace, size_t ws_bytes, void* stream) {
  return kta::decode::launch(Q, Kc, Vc, seqlens, kv_offsets, O, B, Hq, Hkv, D, cache_tokens,
                             max_seqlen, scale, workspace, ws_bytes,
                             static_cast<cudaStream_t>(stream));
}

int kta_decode_gqa_bf16_noalloc(const void* Q, const void* Kc, const void* Vc,
                                const void* seqlens, const void* kv_offsets, void* O, int64_t B,
                                int64_t Hq, int64_t Hkv, int64_t D, int64_t cache_tokens,
                                int64_t max_seqlen, float scale, void* stream) {
  return kta::decode::launch_noalloc(Q, Kc, Vc, seqlens, kv_offsets, O, B, Hq, Hkv, D,
                                     cache_tokens, max_seqlen, scale,
                                     static_cast<cudaStream_t>(stream));
}

}  // extern "C"
