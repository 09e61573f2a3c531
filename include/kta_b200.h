/*
 * libkta_b200 — C ABI of the B200 (sm_100a) kernels behind KTA's kernel cases.
 *
 * Every entry is `extern "C"`, takes device pointers as `const void*` / `void*`, sizes as
 * int64_t and a CUDA stream as `void*` (NULL = the legacy default stream), returns a
 * kta_status code, and is asynchronous on that stream: no host synchronisation happens
 * inside. The caller owns every buffer it passes, and no entry allocates device memory when
 * it is called. The library holds per-device state of its own: a 64-byte device status block
 * written by the kernels' watchdogs, the resolved driver entry point for
 * cuTensorMapEncodeTiled, and one fixed 8 MiB array of device memory (a file-scope
 * __device__ array, held by every GPU that loads the library until the process exits) that
 * only kta_decode_gqa_bf16_noalloc uses. Entries are re-entrant across host threads and
 * streams, except kta_decode_gqa_bf16_noalloc: all its calls share that one array, so calls
 * that overlap on the GPU race and must be serialised by the caller.
 *
 * Reference interfaces these entries replace (paths within kernel-template-agent):
 *   - src/kta/measure/bench.py:94-98 — a `BuiltModule(kind="so")` whose `entry` is called
 *     through ctypes with the LaunchSpec parameters (device addresses as uint64, shape
 *     scalars as int32) and launches by itself. The kta_so_* shims below have exactly that
 *     shape.
 *   - src/kta/backends/harness/run.py:30-77 and src/kta/targets/cudadrv.py:158-177 — the
 *     cubin launch of a TileLang kernel; the kta_* entries are their launch-by-itself
 *     replacements.
 */
#ifndef KTA_B200_H
#define KTA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KTA_ABI_VERSION 1

/* Status codes returned by every entry (and recorded by device watchdogs). */
enum kta_status_code {
  KTA_OK = 0,
  KTA_ERR_INVALID_ARG = 1,    /* null pointer, negative or zero size, bad scale */
  KTA_ERR_UNSUPPORTED = 2,    /* shape or head_dim outside what the kernel handles */
  KTA_ERR_ALIGN = 3,          /* pointer or row stride breaks the 16-byte TMA rule */
  KTA_ERR_LAUNCH = 4,         /* the CUDA launch itself failed */
  KTA_ERR_DEVICE_TIMEOUT = 5, /* a device-side bounded wait expired (see kta_device_status) */
  KTA_ERR_NO_DEVICE = 6,      /* no CUDA device or an sm below 10.0 */
  KTA_ERR_WORKSPACE = 7,      /* workspace missing or smaller than kta_*_workspace_bytes */
  KTA_ERR_CUDA = 8,           /* another CUDA runtime/driver error */
  KTA_ERR_DEVICE_BOUNDS = 9   /* a kernel's own bounds check rejected a device-side value */
};

/* Version of this ABI (KTA_ABI_VERSION of the build). */
int kta_abi_version(void);

/* Static text of a status code. */
const char* kta_status_string(int status);

/* Reads the device status block of the current device into words[0..3]
 * ([0] first error code, [1] site, [2] block, [3] number of failures), after a
 * synchronisation of the device, and clears it when `clear` is nonzero. */
int kta_device_status(uint32_t* words, int clear);

/* Number of SMs of the current device (the persistent grids' size). */
int kta_sm_count(void);

/* Self-test of the device watchdog every kernel's waits go through (no counterpart in the
 * reference, whose kernels have no device-side waits): one thread waits for a barrier phase
 * that nothing completes, gives up after timeout_ns (1 us .. 10 s) of %globaltimer, records
 * KTA_ERR_DEVICE_TIMEOUT with site 0x7F01 in the device status block and returns, leaving the
 * context usable. Asynchronous on `stream`; read the outcome with kta_device_status. */
int kta_watchdog_selftest(uint64_t timeout_ns, void* stream);

/* --- GEMM: C[M,N] = A[M,K] . B[N,K]^T, fp32 accumulate --------------------------------
 * Replaces the TileLang `hgemm` case (perfmodel/testset/gen.py:255-303) and the seed GEMM
 * family (knowledge/seed/families/gemm_fp16_tilelang/gen.py:32-112), launched like
 * src/kta/measure/bench.py:94-98. Row-major A, B, C with leading dimensions lda, ldb, ldc
 * in elements (each a multiple of 8, pointers 16-byte aligned). M = 16..64 runs the
 * swap-AB split-K path (HBM-bound skinny shapes). */
int kta_gemm_bf16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                  int64_t lda, int64_t ldb, int64_t ldc, void* stream);
int kta_gemm_f16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                 int64_t lda, int64_t ldb, int64_t ldc, void* stream);

/* C[M,N] = A[M,K] . B[K,N] with B row-major K x N: the reference's own GEMM case statement
 * `C = A @ B` (knowledge/seed/cases/gemm_fp16.yaml:8-13). Same rules as above. */
int kta_gemm_nn_bf16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                     int64_t lda, int64_t ldb, int64_t ldc, void* stream);
int kta_gemm_nn_f16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                    int64_t lda, int64_t ldb, int64_t ldc, void* stream);

/* --- FP8 block-scaled GEMM -------------------------------------------------------------
 * C[M,N] (bf16) = sum_kb (A[:,kb] . B[:,kb]^T) * sa[m,kb] * sb[n/128,kb], with A [M,K] and
 * B [N,K] e4m3 (row-major), sa [M, ceil(K/128)] fp32 (per 1x128 activation block) and
 * sb [ceil(N/128), ceil(K/128)] fp32 (per 128x128 weight block). Replaces the TileLang
 * `fp8gemm` (perfmodel/testset/gen.py:306-329), which has no scales. K % 16 == 0,
 * N % 8 == 0. */
int kta_gemm_fp8_blockscaled(const void* A, const void* sa, const void* B, const void* sb,
                             void* C, int64_t M, int64_t N, int64_t K, void* stream);

/* --- Causal attention forward -----------------------------------------------------------
 * O = softmax(Q K^T * scale + causal mask) V per (batch, head), LSE = logsumexp of the
 * scaled, masked scores (natural log, fp32). Q, K, V, O bf16 in [B, S, H, D] layout (the
 * layout of perfmodel/testset/gen.py:417-486); LSE fp32 [B, H, S]. D == 128. Replaces the
 * TileLang `fa_forward` (non-causal there). */
int kta_attn_fwd_causal_bf16(const void* Q, const void* K, const void* V, void* O, void* LSE,
                             int64_t B, int64_t H, int64_t S, int64_t D, float scale,
                             void* stream);

/* --- GQA decode attention ---------------------------------------------------------------
 * One query token per sequence: O[b,h,:] = softmax(Q[b,h,:] . K_b^T * scale) V_b with
 * K_b = Kc[kv_offsets[b] : kv_offsets[b] + seqlens[b], h / (Hq/Hkv), :]. Q, O bf16
 * [B, Hq, D]; Kc, Vc bf16 [total_tokens, Hkv, D] (each sequence contiguous); seqlens int32
 * [B] and kv_offsets int64 [B] on the device; cache_tokens = T bounds every
 * kv_offsets[b] + seqlens[b] and max_seqlen every seqlens[b] (checked on the device: a
 * sequence outside them gets a zero output and status KTA_ERR_DEVICE_BOUNDS in the device
 * status block). D == 128, Hq/Hkv <= 16, B <= 2048. The split-KV partials
 * and their log-sum-exp combine (perfmodel/testset/gen.py:493-590) happen in one launch;
 * `workspace` holds the partials and must be at least kta_decode_workspace_bytes(...)
 * bytes, its counters zero before the first call (the kernel leaves them zero).
 * max_seqlen bounds every seqlens[b]. */
size_t kta_decode_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                                  int64_t max_seqlen);
int kta_decode_gqa_bf16(const void* Q, const void* Kc, const void* Vc, const void* seqlens,
                        const void* kv_offsets, void* O, int64_t B, int64_t Hq, int64_t Hkv,
                        int64_t D, int64_t cache_tokens, int64_t max_seqlen, float scale,
                        void* workspace, size_t ws_bytes, void* stream);

/* Allocation-free kta_decode_gqa_bf16. This entry has no counterpart in the reference.
 * Same arguments and results, minus the workspace: the partials and arrival counters live
 * in a fixed 8 MiB array of device memory owned by the library (every GPU that loads the
 * library holds it until the process exits). It is for callers that hand the library only
 * their own input and output buffers and may not allocate device memory themselves: a
 * kernel-case harness that allocates exactly the tensors a case declares and times one
 * launch (an allocation there would synchronise the device inside the timed region), or a
 * host whose device memory belongs to another allocator or was planned up front. Limits:
 * calls whose workspace (kta_decode_workspace_bytes) exceeds 8 MiB return
 * KTA_ERR_UNSUPPORTED; the entry clears the array's counters on `stream` before each launch;
 * all calls share the one array, so calls that overlap on the GPU (other streams or host
 * threads) race and must be serialised by the caller. The first call on a device resolves
 * the array's device address (cudaGetSymbolAddress) with that device current; make that
 * first call before any stream capture. */
int kta_decode_gqa_bf16_noalloc(const void* Q, const void* Kc, const void* Vc,
                                const void* seqlens, const void* kv_offsets, void* O, int64_t B,
                                int64_t Hq, int64_t Hkv, int64_t D, int64_t cache_tokens,
                                int64_t max_seqlen, float scale, void* stream);

/* GEMM with a 4-bit B dequantised in the main loop: C [M, N] f16 = A [M, K] f16 . B^T with
 * B[n, k] = decode(nibble k of Bq[n, :]) * Sc[n, k / group] rounded to f16; Bq [N, K/2] bytes,
 * two elements per byte, the lower nibble first; Sc [N, K/group] f16; fp32 accumulate.
 *   w4a16: decode(x) = x - 8, group a power of two >= 16 (KTA's w4gemm,
 *          perfmodel/testset/gen.py:359-414, group 32 there);
 *   NVFP4: decode = the e2m1 value, group 16 (KTA's nvfp4gemm, gen.py:744-778).
 * K % 64 == 0, K % group == 0, N % 8 == 0; 16-byte aligned A, Bq, C, 2-byte aligned Sc. */
int kta_gemm_w4a16_f16(const void* A, const void* Bq, const void* Sc, void* C, int64_t M,
                       int64_t N, int64_t K, int64_t group, void* stream);
int kta_gemm_nvfp4_f16(const void* A, const void* Bq, const void* Sc, void* C, int64_t M,
                       int64_t N, int64_t K, void* stream);

/* MoE expert GEMM: tokens grouped by expert, T / E rows each; for every expert e,
 * C[e*T/E : (e+1)*T/E, :] = A[e*T/E : (e+1)*T/E, :] . W[e] with A [T, K], W [E, K, N] and C
 * [T, N] row-major f16 or bf16, fp32 accumulate. Replaces KTA's test-set moe_gemm
 * (perfmodel/testset/gen.py:332-356). T % E == 0 and (T / E) % 128 == 0; K % 8 == 0 and
 * N % 8 == 0; 16-byte aligned A, W, C. One launch over every expert. */
int kta_moe_gemm_f16(const void* A, const void* W, void* C, int64_t E, int64_t T, int64_t N,
                     int64_t K, void* stream);
int kta_moe_gemm_bf16(const void* A, const void* W, void* C, int64_t E, int64_t T, int64_t N,
                      int64_t K, void* stream);

/* Row RMSNorm: Y[m, :] = X[m, :] * rsqrt(mean_j X[m, j]^2 + eps) * W, fp32 statistics,
 * X, Y [M, N] and W [N] row-major f16 or bf16. Replaces KTA's test-set rmsnorm
 * (perfmodel/testset/gen.py:662-704, eps 1e-6 there). N % 8 == 0, N <= 16384, 16-byte
 * aligned X, W, Y; eps >= 0. */
int kta_rmsnorm_f16(const void* X, const void* W, void* Y, int64_t M, int64_t N, float eps,
                    void* stream);
int kta_rmsnorm_bf16(const void* X, const void* W, void* Y, int64_t M, int64_t N, float eps,
                     void* stream);

/* Row softmax: Y[m, :] = softmax(X[m, :]) via 2^(x log2 e - max), fp32 max and sum, X, Y
 * [M, N] row-major f16 or bf16. Replaces KTA's test-set softmax
 * (perfmodel/testset/gen.py:781-807). N % 8 == 0, N <= 16384, 16-byte aligned X, Y. */
int kta_softmax_f16(const void* X, void* Y, int64_t M, int64_t N, void* stream);
int kta_softmax_bf16(const void* X, void* Y, int64_t M, int64_t N, void* stream);

/* --- Reference-compatible `so` shims -----------------------------------------------------
 * The exact signature src/kta/measure/bench.py:80-98 calls: pointers as uint64 device
 * addresses, shape scalars as int32, restype None, default stream, the caller synchronises.
 * Errors are recorded in the device status block's host mirror: read them with
 * kta_last_error(). */
void kta_so_gemm_bf16(uint64_t A, uint64_t B, uint64_t C, int32_t M, int32_t N, int32_t K);
void kta_so_gemm_f16(uint64_t A, uint64_t B, uint64_t C, int32_t M, int32_t N, int32_t K);
void kta_so_gemm_nn_f16(uint64_t A, uint64_t B, uint64_t C, int32_t M, int32_t N, int32_t K);
void kta_so_gemm_nn_bf16(uint64_t A, uint64_t B, uint64_t C, int32_t M, int32_t N, int32_t K);
/* the test set's rmsnorm (eps 1e-6) and softmax, f16, with its (X, W, Y, M, N) / (X, Y, M, N)
 * parameters (perfmodel/testset/gen.py:662-704, :781-807) */
void kta_so_rmsnorm_f16(uint64_t X, uint64_t W, uint64_t Y, int32_t M, int32_t N);
/* the test set's w4gemm (group 32) and nvfp4gemm, with their (A, Bq, Sc, C) tensors */
void kta_so_w4gemm_f16(uint64_t A, uint64_t Bq, uint64_t Sc, uint64_t C, int32_t M, int32_t N,
                       int32_t K);
void kta_so_nvfp4gemm_f16(uint64_t A, uint64_t Bq, uint64_t Sc, uint64_t C, int32_t M, int32_t N,
                          int32_t K);
/* the test set's moe_gemm, f16, with its (A, W, C) tensors and (E, T, N, K) sizes */
void kta_so_moe_gemm_f16(uint64_t A, uint64_t W, uint64_t C, int32_t E, int32_t T, int32_t N,
                         int32_t K);
void kta_so_softmax_f16(uint64_t X, uint64_t Y, int32_t M, int32_t N);

/* Status of the last kta_so_* call on this host thread. */
int kta_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* KTA_B200_H */
