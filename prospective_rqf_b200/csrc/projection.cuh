// Complex projection GEMM of the Pure RQF block on the 5th-generation tensor
// cores (tcgen05 + TMA + TMEM), in split TF32:
//
//   out[j, n] = sum_k op(W)[j, k] * X[k, n]   (+ acc[j, n])          complex64
//
// op(W) = W gives the block projection z = W h (rqf_models/backbones/rqf/
// pure.py:223, a torch.matmul on the (d_model, batch*time) view); op(W) = W^H
// gives its input cotangent W^H gz, and `acc` folds in the skip cotangent.
// X is (K, N) with N contiguous: the (F,B,T) activations with N = B*T.
//
// Real formulation.  A' is the (2M x K) real matrix whose rows alternate
// Re op(W)[j,:] and Im op(W)[j,:]; X' = view_as_real(X) is (K x 2N) with
// columns alternating Re and Im.  P = A' X' holds the four real products of
// each complex product, and
//     Re out[j,n] = P[2j, 2n] - P[2j+1, 2n+1],   Im out[j,n] = P[2j, 2n+1] + P[2j+1, 2n].
// Rows 2j and 2j+1 of a tile sit in adjacent TMEM lanes, i.e. adjacent
// threads of one epilogue warp, which combine them with shuffles.
//
// Precision.  tcgen05.mma kind::tf32 converts its fp32 operands to TF32 by
// truncation (round toward zero; measured on B200 by an in-bounds MMA of
// values with low mantissa bits set against exact ones).  So the raw fp32
// value v already serves as hi = trunc_tf32(v), and only lo =
// rna_tf32(v - trunc_tf32(v)) is materialised; the tile accumulates
// A_hi X_hi + A_hi X_lo + A_lo X_hi in fp32: about 21 significant bits per
// operand against 10 for a single TF32 product, i.e. fp32-comparable (the
// fp32 SIMT complex GEMM it replaces keeps 24).  A' is split once per call
// by proj_prep_kernel; X' is split in shared memory by four transform warps
// right after its TMA load (writing only the lo part), so the activations
// cross HBM once.
//
// CTA pairs (clusters of 2, one CTA per SM, persistent over pair tiles of
// 256 A' rows x 256 X' columns): each tcgen05.mma.cta_group::2 (M = 256,
// N = 256, K = 8) is issued by rank 0 and reads each CTA's half of A (its
// 128 rows) and of B (its 128 columns) at the same shared-memory offsets;
// each CTA's TMEM holds its 128 rows of D.  Per CTA:
//   warp 0      TMA producer: A_hi, A_lo (K-major, 64-byte swizzle) and its
//               X' columns (MN-major, 128-byte swizzle of 32-byte atoms)
//   warp 1      TMEM allocation (both CTAs) and, in rank 0, the MMA issuer
//   warps 2..5  epilogue: TMEM -> registers, complex combine, staged through
//               shared memory into full-line row stores (+acc)
//   warps 6..9  transform: X' stage -> lo part (the raw stage is the hi part)
// Six shared-memory stages of K = 16 (five of 40 KB in the real-output
// form) and two TMEM accumulators (2 x 256
// columns), so the epilogue of one tile overlaps the MMAs of the next.  The
// peer's transform and epilogue warps arrive on the leader's barriers through
// the cluster window; the leader's commits arrive on both CTAs' barriers.
// Variants: a real X (rqf_projection_real: samples, not (Re, Im) pairs) and a
// real output (rqf_projection_real_out: Re(op(W) X) only, X split into its Re
// and Im planes by the transform).  Every mbarrier wait is bounded in time;
// on expiry the kernel latches RQF_ERR_PIPELINE_TIMEOUT, every role stops,
// in-flight copies and MMAs are waited for (bounded) and the TMEM is freed
// before exit.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fbt_scan.cuh"
#include "rqf_common.cuh"

namespace rqf {
namespace proj {

constexpr int kBM = 128;              // A' rows per CTA (TMEM lanes)
constexpr int kPairM = 2 * kBM;       // A' rows per CTA-pair tile: M of the two-SM MMA
constexpr int kBN = 256;              // X' columns per pair tile: N of the MMA
constexpr int kBNh = kBN / 2;         // X' columns each CTA of the pair stages
constexpr int kBK = 16;               // K per stage: one 64-byte swizzle row of fp32
constexpr int kUmmaK = 8;             // K of one tcgen05.mma kind::tf32
constexpr int kStages = 6;
constexpr int kAccBufs = 2;
constexpr int kTmemCols = kBN * kAccBufs;  // 512: the whole TMEM of the SM
constexpr int kThreads = 320;
constexpr int kNBlocks = kBNh / 32;   // 32-column (128-byte) blocks of a CTA's X' stage

constexpr int kABytes = kBM * kBK * 4;            // 8 KB, one of A_hi / A_lo
constexpr int kBBytes = kBK * kBNh * 4;           // 8 KB, one of X_hi / X_lo
constexpr int kStageBytes = 2 * kABytes + 2 * kBBytes;  // 32 KB
constexpr int kTxBytes = 2 * kABytes + kBBytes;   // bytes the TMA lands per stage
constexpr int kBarBytes = 256;
// Epilogue staging: each epilogue warp turns its 16 output rows x 32 samples
// into full-line row stores through 4 KB of shared memory.
constexpr int kStagingBytes = 4 * 4096;
// Real-output mode (Re(op(W) x) as float32, for the readout's hidden layer):
// a stage also holds the raw x tile, 8 complex k rows x 128 samples (Re, Im
// interleaved, no swizzle), which the transform splits into the Re and Im
// planes of B; A = [Re op(W) | -Im op(W)] per k-block of 8 complex k.
constexpr int kRawXBytes = 8 * kBNh * 2 * 4;     // 8 KB
constexpr int kRawXOff = kStageBytes;            // after the four operand tiles
// Scan modes (kScan: 1 the block forward, 2 its backward): each epilogue
// warp stages its two outputs (16 rows x 128 B each, in the 128-byte swizzle
// of the TMA stores, so 1024-byte aligned: the staging comes right after the
// stages) and the tile's entry slots.
constexpr int kScanFwd = 1, kScanBwd = 2;
constexpr int kScanWarpStaging = 3 * 2048;
// The backward scan mode also gives each epilogue warp a two-slot ring of
// TMA-loaded chunks of its rows of z and acc (per slot 16 rows x 128 B of
// each, in the 128-byte swizzle), and runs one operand stage fewer to make
// room for it.
constexpr int kRingSlotBytes = 4096;
constexpr int kRingWarpBytes = 2 * kRingSlotBytes;
template <bool kRealOut, int kScan = 0>
struct ProjLayout {
  static constexpr int kStages = (kRealOut || kScan == kScanBwd) ? 5 : 6;
  static constexpr int kStageBytes = kRealOut ? ::rqf::proj::kStageBytes + kRawXBytes
                                              : ::rqf::proj::kStageBytes;  // 40 / 32 KB
  static constexpr int kWarpStaging = kScan ? kScanWarpStaging : kStagingBytes / 4;
  static constexpr int kRingBytes = kScan == kScanBwd ? 4 * kRingWarpBytes : 0;
  // scan modes: staging, ring, barriers; otherwise barriers then staging
  // staging (1024-byte aligned for the TMA tensor stores), ring, barriers
  static constexpr int kStagingOff = kStages * kStageBytes;
  static constexpr int kRingOff = kStages * kStageBytes + 4 * kWarpStaging;
  static constexpr int kBarOff = kRingOff + kRingBytes;
  static constexpr int kSmemBytes =
      kStages * kStageBytes + kBarBytes + 4 * kWarpStaging + kRingBytes + 1024;  // + alignment slack
};
constexpr int kSmemBytes = ProjLayout<false>::kSmemBytes;
constexpr int kScanSmemBytes = ProjLayout<false, kScanFwd>::kSmemBytes;
constexpr int kScanBwdSmemBytes = ProjLayout<false, kScanBwd>::kSmemBytes;
static_assert(ProjLayout<false, kScanBwd>::kRingOff % 1024 == 0,
              "the ring's swizzled slots need 1024-byte alignment");
static_assert(kScanBwdSmemBytes <= 227 * 1024, "shared memory per CTA");

constexpr int kErrPipelineTimeout = 7;            // RQF_ERR_PIPELINE_TIMEOUT
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s per wait

// Where the first expired wait of the projection pipeline gave up (0 = none):
// 1 producer/empty, 2 transform/full, 3 MMA/accumulator-drained, 4 MMA/ready,
// 5 epilogue/accumulator-full, 6 shutdown drain, 7 scan epilogue/link record
// of the tile before along its chain, 8 backward scan epilogue/ring load.
// Read by rqf_projection_timeout_site().
__device__ int g_proj_timeout_site;

struct Params {
  float2 *out;
  const float2 *acc;   // may be null
  long long M;         // complex output rows
  long long N;         // complex samples
  int K;               // complex reduction length
  int m_pairs, n_tiles, k_blocks;  // pair tiles: kPairM A' rows x kBN X' columns
  long long num_tiles;
  int a_rows_pad;      // rows of the hi half of the split A' buffer (a multiple of kPairM)
  int real_x;          // X real (K x N): columns are samples, not (Re, Im) pairs
  float *out_real;     // real-output mode: Re(op(W) x), float32 (M x N)
  // Scan mode (proj_kernel<false, true>): the epilogue also runs the Pure RQF
  // block's two-tap scan along each output row (see ScanParams).
  int scan;
  // Accumulate in place (complex X, out == acc): the epilogue adds its tile
  // into out with a TMA reduce-add through ScanParams::tmZ (out as M rows x
  // 2N floats) instead of loading acc, so no epilogue warp waits on it.
  int inplace;
};

// The block scan fused into the projection's epilogue: out row j of the
// (F,B,T) layout is filter j, N = B*T samples with T contiguous.  Per row,
//   y[t] = c1 y[t-1] + tap0 z[t] + tap1 z[t-1],  act = split-ReLU(y) or y,
//   out = act + skip,
// computed exactly as fbt_fwd_rows_kernel computes it (same drive and
// recurrence operations, 8 samples sequentially from their entry), so the
// (F,B,T) backward replays the same states from the entries saved here.
//
// The backward mode (kScanBwd) runs the same block's scan VJP in the epilogue
// of its input-cotangent GEMM: out = W'^H gz' + acc is the cotangent g of
// the block below (W' and gz' those of the block above, acc the skip's
// cotangent), and the epilogue turns g into that block's gz (see
// scan_bwd_epilogue).  Fields in that mode: tmZ maps out (the GEMM output),
// tmAct maps grad_z; c1, tap0, tap1, zin, carries and fuse_act belong to the
// scanned block (its saved context); skip and act are unused.
struct ScanParams {
  CUtensorMap tmZ, tmAct;          // out (z) and act as (M rows, 2N floats), 16 x 32 boxes, 128-B swizzle
  const float2 *c1, *tap0, *tap1;  // (M,)
  const float2 *skip;              // (M, N) or null
  float2 *act;                     // (M, N) output
  float2 *carries;                 // fbt_slot layout of the (F,B,T) kernels
  const float2 *zin;               // backward: the scanned block's z (M, N)
  CUtensorMap tmZin, tmAcc;        // backward: zin and p.acc, as tmZ (TMA loads into the ring)
  // backward: (M * batch rows, tiles_per_row, 3) per-tile sums of
  // conj(y[t-1]) d, conj(z) d, conj(z[t-1]) d, summed by reduce_partials_kernel
  float2 *partials;
  int reverse;                     // backward: each chain runs from the end of its batch row
  float4 *link;                    // (num_tiles, 2 ranks, 64 rows): {y, z} at a tile's end
  // (num_tiles, 2 ranks, 4 epilogue warps) link-published flags, then one
  // abort word; all zeroed before the launch
  unsigned *flags;
  long long T;                     // samples per batch row (a multiple of 128)
  int batch;                       // N / T
  int tiles_per_row;               // T / 128: pair tiles of one (row block, batch) chain
  int chains;                      // m_pairs * batch
  int fbt_ntiles;                  // ceil(T / 2048): tiles of the (F,B,T) saved context
  int fuse_act;
};

// ------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// try_wait with a suspend-time hint: a waiting warp sleeps in hardware (up to
// the hint, in ns) instead of re-issuing the poll, leaving issue slots to
// the transform and epilogue warps.
constexpr uint32_t kSuspendHintNs = 1000000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of `parity` to complete.  Returns false (and
// raises the CTA's abort flag, latching the error once) when the time limit
// passes or another role has already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                          int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31u) == 0u) {
      if (*abort) return false;
      if (global_ns() - t0 > kWaitLimitNs) {  // each poll sleeps at most kSuspendHintNs
        latch_error(kErrPipelineTimeout);
        atomicCAS(&g_proj_timeout_site, 0, site);
        *abort = 1;
        return false;
      }
    }
  }
}
// Wait used while shutting down: bounded, ignores the abort flag.
__device__ __forceinline__ void mbar_drain(uint64_t *bar, uint32_t parity) {
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) {
      latch_error(kErrPipelineTimeout);
      atomicCAS(&g_proj_timeout_site, 0, 6);
      return;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
// TMA tensor store of a shared-memory box, tracked by this thread's bulk
// groups: commit after issuing, wait (.read: until the source may be
// overwritten; plain: until the writes are complete).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x,
                                             int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
// TMA tensor reduce of a shared-memory box into global memory: element-wise
// fp32 add (each element of the box is added once).
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *map, const void *src, int x,
                                                  int y) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// generic-proxy shared-memory writes -> visible to the async proxy (TMA)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// ------------------------------------------------------------ CTA pair
// The two CTAs of a cluster (ranks 0 and 1) run on the two SMs of one TPC and
// share each tcgen05.mma.cta_group::2: rank 0 (the leader) issues it, each
// CTA holds its half of A (128 rows) and of B (N/2 columns) at the same
// shared-memory offsets, and each CTA's TMEM receives its 128 rows of D.
// The peer reaches the leader's barriers through the cluster window; the
// leader's commits arrive on both CTAs' barriers, one commit per barrier.
__device__ __forceinline__ uint32_t pair_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t pair_index() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t pair_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// Address of `local`'s counterpart in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void *local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(caddr)
               : "memory");
}
// Every thread of both CTAs.
__device__ __forceinline__ void pair_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_commit_pair(uint32_t caddr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   caddr)
               : "memory");
}
__device__ __forceinline__ void tc_mma_pair_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// TMEM of the pair: one warp of each CTA (the same warp index) allocates and
// frees together.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free_pair(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols)
               : "memory");
}

// 32 lanes x 32 consecutive fp32 columns: thread i of the warp receives
// columns [col, col+32) of TMEM lane (lane base + i).
__device__ __forceinline__ void tc_ld_32x32b_x32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// The inverse: thread i writes v to columns [col, col+32) of lane (base + i).
// Completion is awaited with tcgen05.wait::st.
__device__ __forceinline__ void tc_st_32x32b_x32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ float tf32_rna(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return __uint_as_float(r);
}
// The low part of the split: v minus the TF32 value the tensor core reads
// for v (its truncation), rounded to TF32 so that it is read exactly.
__device__ __forceinline__ float tf32_lo(float v) {
  return tf32_rna(v - __uint_as_float(__float_as_uint(v) & 0xffffe000u));
}

// Shared-memory matrix descriptor of tcgen05.mma: start, leading and stride
// byte offsets in 16-byte units, descriptor version 1, swizzle mode.
//   kSwizzle64B        (4): 16-byte chunks XOR-ed over 8 rows of 64 bytes —
//                           the K-major A' tile (TMA CU_TENSOR_MAP_SWIZZLE_64B);
//   kSwizzle128BBase32 (1): 32-byte chunks XOR-ed over 4 rows of 128 bytes —
//                           what an MN-major 32-bit operand must use (the X'
//                           tile; TMA CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B).
constexpr uint64_t kSwizzle64B = 4, kSwizzle128BBase32 = 1;
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                              uint64_t swizzle) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (swizzle << 61);
}

// Instruction descriptors (kind::tf32, D fp32): M = 256 (the CTA pair), N = 256.
// kIdesc: A K-major, B MN-major (the projection's X').  kIdescKK: both
// K-major (the weight gradient's h' rows).
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (0u << 15) | (1u << 16) |
                            ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kPairM >> 4) << 24);
constexpr uint32_t kIdescKK = (1u << 4) | (2u << 7) | (2u << 10) | (0u << 15) | (0u << 16) |
                              ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kPairM >> 4) << 24);

// ------------------------------------------------------------ weight split
// A' rows alternate Re and Im of op(W)[j,:]; hi in rows [0, rows_pad), lo in
// rows [rows_pad, 2 rows_pad) of a (2 rows_pad x k_pad) fp32 buffer, padding
// zero.  op(W) = W for W (M x K); op(W) = W^H for W (K x M).
__global__ void proj_prep_kernel(const float2 *__restrict__ W, float *__restrict__ a_split,
                                 long long M, int K, int rows_pad, int k_pad, int conj_t) {
  const long long total = (long long)rows_pad * k_pad;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / k_pad;
    const int k = (int)(i - r * k_pad);
    float v = 0.f;
    if (r < 2 * M && k < K) {
      const long long j = r >> 1;
      if (!conj_t) {
        const float2 w = W[j * K + k];
        v = (r & 1) ? w.y : w.x;
      } else {
        const float2 w = W[(long long)k * M + j];
        v = (r & 1) ? -w.y : w.x;
      }
    }
    a_split[i] = v;  // read as trunc_tf32(v) by the tensor core
    a_split[total + i] = tf32_lo(v);
  }
}

// Real-output A: row j, k-block b (16 columns) = [Re W[j, 8b..8b+8) |
// -Im W[j, 8b..8b+8)], hi in rows [0, rows_pad), lo in [rows_pad, 2 rows_pad).
__global__ void proj_prep_real_out_kernel(const float2 *__restrict__ W, float *__restrict__ a_split,
                                          long long M, int K, int rows_pad, int k3_pad) {
  const long long total = (long long)rows_pad * k3_pad;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / k3_pad;
    const int c = (int)(i - r * k3_pad);
    const int e = c & 15, k = (c >> 4) * 8 + (e & 7);
    float v = 0.f;
    if (r < M && k < K) {
      const float2 w = W[r * K + k];
      v = e < 8 ? w.x : -w.y;
    }
    a_split[i] = v;
    a_split[total + i] = tf32_lo(v);
  }
}

// ------------------------------------------------------------ main kernel
// Pair tile t covers A' rows [mp*256, mp*256+256) and X' columns
// [nt*256, nt*256+256); the pair tiles of one X' column block are neighbours
// (mp fastest), so the block is read from HBM once and from L2 after.
// In scan mode the tiles run position-major over the (row block, batch)
// chains instead: the pair tiles that run at the same time belong to different
// chains, so a tile's predecessor along its chain (the tile `chains` earlier:
// the one before it in time, or after it in the backward) has normally
// finished before its epilogue needs the predecessor's end state.
__device__ __forceinline__ void tile_coords(long long tile, const Params &p, int &mp, int &nt,
                                            const ScanParams *sp = nullptr) {
  if (sp != nullptr && p.scan) {
    const long long step = tile / sp->chains;  // position along the chain
    const int ch = (int)(tile - step * sp->chains);
    const long long pos = sp->reverse ? sp->tiles_per_row - 1 - step : step;
    mp = ch % p.m_pairs;
    nt = (int)((long long)(ch / p.m_pairs) * sp->tiles_per_row + pos);
    return;
  }
  mp = (int)(tile % p.m_pairs);
  nt = (int)(tile / p.m_pairs);
}

// Byte offset of element (column c, row k) of an MN-major 32-bit operand tile
// of kBK rows in the 128-byte swizzle of 32-byte atoms: 32-column blocks of
// kBK rows x 128 bytes, 32-byte atom (c & 31) >> 3 of row k at that ^ (k & 3).
__device__ __forceinline__ uint32_t mn32_offset(int c, int k) {
  return (uint32_t)((c >> 5) * (kBK * 128) + k * 128 + ((((c & 31) >> 3) ^ (k & 3)) << 5) +
                    ((c & 7) << 2));
}

// ------------------------------------------------------------ scan epilogue
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned *p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(unsigned *p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_u32(unsigned *p, unsigned v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait of one epilogue warp for the link record of the tile before
// its own along time.  False when the time limit passes (error latched) or
// when this CTA or any other has aborted; either way the launch-wide abort
// word is raised so that no other waiter runs into its own time limit.
__device__ __forceinline__ bool scan_link_wait(const unsigned *flag, unsigned *abort_word,
                                               volatile int *abort) {
  const unsigned long long t0 = global_ns();
  unsigned ns = 64;
  for (;;) {
    if (ld_acquire_u32(flag) != 0u) return true;
    if (*abort || ld_relaxed_u32(abort_word) != 0u) break;
    if (global_ns() - t0 > kWaitLimitNs) {
      latch_error(kErrPipelineTimeout);
      atomicCAS(&g_proj_timeout_site, 0, 7);
      break;
    }
    __nanosleep(ns);
    ns = ns < 1024u ? 2u * ns : 1024u;
  }
  *abort = 1;
  st_relaxed_u32(abort_word, 1u);
  return false;
}

// A scan-mode tile's saved entries: the 16 consecutive slots of each of the
// warp's 16 rows of the (F,B,T) context, staged in `ent` ([16 rows][16
// slots], 16-byte chunk k of row r at k ^ (r & 7)), written as one 128-byte
// piece per row.
__device__ __forceinline__ void scan_save_entries(const float2 *ent, const Params &p,
                                                  const ScanParams &sp, long long jw0, int bidx,
                                                  int pos, long long tfirst, int lane) {
  __syncwarp();
  const long long jt = tfirst / kFbtTile;
  const int s0 = (int)(tfirst - jt * kFbtTile) / kFbtK;
  const float4 *ent4 = reinterpret_cast<const float4 *>(ent);
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int e4 = it * 32 + lane;
    const int rr = e4 >> 3, k = e4 & 7;
    const long long jj = jw0 + rr;
    if (jj < p.M)
      *reinterpret_cast<float4 *>(
          sp.carries + fbt_slot(jj * sp.batch + bidx, sp.fbt_ntiles, (int)jt) + s0 + 2 * k) =
          ent4[rr * 8 + (k ^ (rr & 7))];
  }
  // The slots past T of the row's last context tile: zero, so that the
  // backward's replay of the padded samples stays finite.
  if (pos == sp.tiles_per_row - 1) {
    const long long jl = (sp.T - 1) / kFbtTile;
    const int used = (int)(sp.T - jl * kFbtTile) / kFbtK;  // T % 128 == 0: even
    const int pairs = (kFbtSlots - used) / 2;
    for (int i = lane; i < 16 * pairs; i += 32) {
      const int rr = i / pairs, k = i - rr * pairs;
      const long long jj = jw0 + rr;
      if (jj < p.M)
        *reinterpret_cast<float4 *>(sp.carries +
                                    fbt_slot(jj * sp.batch + bidx, sp.fbt_ntiles, (int)jl) +
                                    used + 2 * k) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  __syncwarp();  // staging reads done before the next tile writes
}

// One epilogue warp's share of a scan-mode pair tile: 16 filter rows (lane
// pair 2r, 2r+1 holds row jw0 + r) x the tile's 128 samples, which lie in one
// batch row because T is a multiple of 128.  Eight chunks of 16 samples,
// the even lane's 8 then the odd lane's 8; per chunk:
//   z        combined from the TMEM products as in the plain epilogue,
//            staged (128-byte swizzle) and written by a TMA tensor store to
//            p.out (the (F,B,T) backward reads it);
//   drive    b[k] = tap0 z[k] + tap1 z[k-1] (fbt_drive, as every (F,B,T)
//            kernel computes it);
//   entry    the even lane enters with the row's running state E and folds
//            its 8 drives; the odd lane enters with that result;
//   outputs  both lanes run y = c1 y + b[k] from their own entry (the
//            operations that the (F,B,T) backward replays from the saved
//            entry, so its split-ReLU mask is this one), act = split-ReLU(y)
//            or y, plus skip, staged and written by a TMA tensor store to
//            sp.act.
// The skip lines of the tile are prefetched into L2 when it starts and each
// lane loads its own 8 samples one chunk ahead, so no load waits on HBM.
// The two staging buffers are reused once the bulk store that read them has
// finished reading (bulk groups: z then act per chunk, waited with one group
// left outstanding).  Every lane's entry is the saved context slot of its 8
// samples; the 16 slots of each row are staged and written as one 128-byte
// piece per tile.  The state entering the tile, {y, z} at the sample before
// it, is the link record that the tile before it along time (tile - chains)
// published; at the end of the tile this one publishes its own.  False on an
// abort.
__device__ __forceinline__ bool scan_epilogue(uint32_t tbase, float4 *stage, const Params &p,
                                              const ScanParams &sp, long long tile, int mp,
                                              int nt, int rank, int quarter, int lane,
                                              volatile int *abort) {
  const bool odd = (lane & 1) != 0;
  const int r_own = lane >> 1;
  const long long jw0 = ((long long)mp * kPairM + (long long)rank * kBM + quarter * 32) >> 1;
  const long long jrow = jw0 + r_own;
  const bool row_ok = jrow < p.M;
  const bool warp_ok = jw0 < p.M;  // some row of the warp's 16 exists
  const int bidx = nt / sp.tiles_per_row;
  const int pos = nt - bidx * sp.tiles_per_row;
  const long long tfirst = (long long)pos * (kBN / 2);  // first sample in the batch row
  const long long n0 = (long long)nt * (kBN / 2);       // first sample in N
  const float2 lam = row_ok ? __ldg(sp.c1 + jrow) : cz();
  const float2 tap0 = row_ok ? __ldg(sp.tap0 + jrow) : cz();
  const float2 tap1 = row_ok ? __ldg(sp.tap1 + jrow) : cz();
  unsigned *abort_word = sp.flags + p.num_tiles * 8;
  const bool has_skip = sp.skip != nullptr;
  const bool lane_skip = has_skip && row_ok;
  // this lane's 8 skip samples of chunk c: the 64 bytes at skrow + 8 c
  const float4 *skrow =
      lane_skip ? reinterpret_cast<const float4 *>(sp.skip + jrow * p.N + n0 + (odd ? 8 : 0))
                : nullptr;
  if (has_skip && lane < 16 && jw0 + lane < p.M)  // the tile's 1 KB of each row, into L2
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], 1024;" ::"l"(sp.skip + (jw0 + lane) * p.N + n0)
                 : "memory");
  float4 skn[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    skn[i] = lane_skip ? __ldg(skrow + i) : make_float4(0.f, 0.f, 0.f, 0.f);

  float2 E = cz(), zl = cz();  // y and z at the sample before the chunk
  if (pos > 0) {
    const long long pred = (tile - sp.chains) * 2 + rank;
    const bool ok = scan_link_wait(sp.flags + pred * 4 + quarter, abort_word, abort);
    if (!__all_sync(0xffffffffu, ok)) return false;
    const float4 l = __ldcg(sp.link + pred * 64 + quarter * 16 + r_own);
    E = make_float2(l.x, l.y);
    zl = make_float2(l.z, l.w);
  }
  float4 *zst = stage;                                    // z staging, 16 rows x 128 B
  float4 *ast = stage + 128;                              // act staging
  float2 *ent = reinterpret_cast<float2 *>(stage + 256);  // [16 rows][16 slots], swizzled

#pragma unroll 1
  for (int c = 0; c < kBN / 32; ++c) {
    const long long nbase = n0 + c * 16;
    float4 sk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) sk[i] = skn[i];
    if (lane_skip && c + 1 < kBN / 32) {
#pragma unroll
      for (int i = 0; i < 4; ++i) skn[i] = __ldg(skrow + 8 * (c + 1) + i);
    }
    float v[32];
    tc_ld_32x32b_x32(tbase + (uint32_t)(c * 32), v);
    float r[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) r[i] = __shfl_xor_sync(0xffffffffu, odd ? v[i] : v[16 + i], 1);
    float2 z[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float pr_re = odd ? r[2 * t] : v[2 * t];
      const float pr_im = odd ? r[2 * t + 1] : v[2 * t + 1];
      const float pi_re = odd ? v[16 + 2 * t] : r[2 * t];
      const float pi_im = odd ? v[16 + 2 * t + 1] : r[2 * t + 1];
      z[t] = make_float2(pr_re - pi_im, pr_im + pi_re);
    }
    if (lane == 0) bulk_wait_read<1>();  // the previous z store has read its staging
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q)
      zst[r_own * 8 + (((odd ? 4 : 0) + q) ^ (r_own & 7))] =
          make_float4(z[2 * q].x, z[2 * q].y, z[2 * q + 1].x, z[2 * q + 1].y);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (warp_ok) tma_store_2d(&sp.tmZ, zst, (int)(2 * nbase), (int)jw0);
      bulk_commit();
    }

    // drives; the odd lane's z before its first sample is the even lane's last
    const float2 zx = shfl_xor2(z[7], 1);
    float2 bd[8];
    fbt_drive<8>(tap0, tap1, z, odd ? zx : zl, bd);
    zl = odd ? z[7] : zx;  // both lanes: z at the chunk's last sample
    // entries: the even lane's is E, the odd lane's the even lane's fold of E
    float2 y = E;
#pragma unroll
    for (int k = 0; k < 8; ++k) y = c_fma(lam, y, bd[k]);
    const float2 yx = shfl_xor2(y, 1);
    float2 e = odd ? yx : E;
    ent[r_own * 16 + ((c ^ (r_own & 7)) << 1) + (odd ? 1 : 0)] = e;
    float2 o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      e = c_fma(lam, e, bd[k]);
      o[k] = sp.fuse_act ? c_relu(e) : e;
    }
    const float2 ex = shfl_xor2(e, 1);
    E = odd ? e : ex;  // both lanes: y at the chunk's last sample

    if (lane == 0) bulk_wait_read<1>();  // the previous act store has read its staging
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q)
      ast[r_own * 8 + (((odd ? 4 : 0) + q) ^ (r_own & 7))] =
          make_float4(o[2 * q].x + sk[q].x, o[2 * q].y + sk[q].y, o[2 * q + 1].x + sk[q].z,
                      o[2 * q + 1].y + sk[q].w);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (warp_ok) tma_store_2d(&sp.tmAct, ast, (int)(2 * nbase), (int)jw0);
      bulk_commit();
    }
  }

  // publish {y, z} at the tile's last sample for the tile after it, before
  // the saved entries: the tile after it along time waits on this, and the
  // fence below then waits for this one store only
  if (pos + 1 < sp.tiles_per_row) {
    const long long me = tile * 2 + rank;
    if (odd) sp.link[me * 64 + quarter * 16 + r_own] = make_float4(E.x, E.y, zl.x, zl.y);
    __threadfence();
    __syncwarp();
    if (lane == 0) st_release_u32(sp.flags + me * 4 + quarter, 1u);
  }
  scan_save_entries(ent, p, sp, jw0, bidx, pos, tfirst, lane);

  return true;
}

// Ring of one epilogue warp in the backward scan mode.  The chunks the warp
// consumes form one sequence over its tiles: chunk c of its j-th tile is
// k = 8 j + 7 - c, lands in slot k & 1 and completes phase (k >> 1) & 1 of
// that slot's barrier.  Lane 0 issues chunk k + 2 once every lane has used
// chunk k, so each load has a chunk's work to land.
struct ScanRing {
  uint8_t *base;      // two slots of kRingSlotBytes: z rows (2 KB), then acc rows (2 KB)
  uint64_t *bar;      // one barrier per slot
  long long npairs;
  uint32_t issued;    // lane 0: chunks whose loads were issued
  uint32_t consumed;  // chunks used
};

// Lane 0: issue the TMA loads of chunk k, the 16 rows from y x 16 samples
// from x / 2 of z and of acc, in the layout of the staging.
__device__ __forceinline__ void ring_issue(ScanRing &r, uint32_t k, const Params &p,
                                           const ScanParams &sp, int x, int y) {
  uint8_t *slot = r.base + (k & 1) * kRingSlotBytes;
  uint64_t *bar = r.bar + (k & 1);
  const bool acc = p.acc != nullptr;
  mbar_expect_tx(bar, acc ? 4096u : 2048u);
  tma_load_2d(slot, &sp.tmZin, bar, x, y);
  if (acc) tma_load_2d(slot + 2048, &sp.tmAcc, bar, x, y);
  r.issued = k + 1;
}
// Where chunk c of tile t starts: x (floats along the rows) and y (the
// warp's first row); false past the last tile.
__device__ __forceinline__ bool ring_coords(long long t, int c, const Params &p,
                                            const ScanParams &sp, int rank, int quarter, int &x,
                                            int &y) {
  if (t >= p.num_tiles) return false;
  int mp, nt;
  tile_coords(t, p, mp, nt, &sp);
  y = (int)(((long long)mp * kPairM + (long long)rank * kBM + quarter * 32) >> 1);
  x = (int)(2 * ((long long)nt * (kBN / 2) + 16 * c));  // 128-byte aligned
  return true;
}

// One epilogue warp's share of a backward-mode pair tile: 16 rows (lane pair
// 2r, 2r+1 holds row jw0 + r) x the tile's 128 samples of one batch row,
// in chunks of 16 samples from the tile's end to its start (the even lane
// holds the chunk's first 8 samples, the odd lane the last 8).  Per chunk:
//   g        the GEMM output combined from the TMEM products, plus acc (the
//            skip's cotangent), staged and written by a TMA tensor store to
//            p.out: the block's output cotangent, and the acc of the next
//            GEMM down;
//   replay   the drive b[k] = tap0 z[k] + tap1 z[k-1] (fbt_drive) and
//            y = c1 y + b[k] from the lane's saved entry state: the
//            forward's own operations, so the states and the split-ReLU mask
//            are the forward's bit for bit;
//   adjoint  d[t] = mask(y[t]) g[t] + conj(c1) d[t+1]: the odd lane's fold of
//            its 8 samples from D (d after the chunk) is the even lane's
//            entry; then both lanes run their samples, giving
//            grad_z[t] = conj(tap0) d[t] + conj(tap1) d[t+1] (staged, TMA
//            tensor store through tmAct) and the sums conj(y[t-1]) d[t],
//            conj(z[t]) d[t], conj(z[t-1]) d[t] of the coefficient
//            gradients, on paired fp32 FMAs as in fbt_bwd_rows_kernel.
// z and acc arrive through the warp's ring (TMA loads, two chunks ahead):
// per-lane global loads of 16 rows each would queue behind the tensor core's
// shared-memory traffic.  The z sample before the even lane's first one is
// the odd lane's last of the next chunk in the ring (one load per tile before
// the tile's first sample).  D entering the tile is d at the first sample
// of the tile after it, published by that tile (the one `chains` earlier in
// this launch) as its link record; zero at the end of a batch row.  The tile
// publishes d at its own first sample at the end.  Its three sums per row go
// to sp.partials[(row, tile)].  False on an abort.
__device__ __forceinline__ bool scan_bwd_epilogue(uint32_t tbase, float4 *stage, const Params &p,
                                                  const ScanParams &sp, long long tile, int mp,
                                                  int nt, int rank, int quarter, int lane,
                                                  ScanRing &ring, volatile int *abort) {
  const bool odd = (lane & 1) != 0;
  const int r_own = lane >> 1;
  const long long jw0 = ((long long)mp * kPairM + (long long)rank * kBM + quarter * 32) >> 1;
  const long long jrow = jw0 + r_own;
  const bool row_ok = jrow < p.M;
  const bool warp_ok = jw0 < p.M;  // some row of the warp's 16 exists
  const int bidx = nt / sp.tiles_per_row;
  const int pos = nt - bidx * sp.tiles_per_row;     // the tile's place in its batch row
  const long long step = tile / sp.chains;           // its place along the chain (reversed)
  const long long tfirst = (long long)pos * (kBN / 2);
  const long long n0 = (long long)nt * (kBN / 2);
  unsigned *abort_word = sp.flags + p.num_tiles * 8;
  // The replay needs every thread's entry state in the saved context.
  if (lane == 0 && __ldg(sp.carries + fbt_marker(p.M * sp.batch, sp.fbt_ntiles)).x != 1.f)
    latch_error(5);  // RQF_ERR_ARGUMENT
  const float2 lam = row_ok ? __ldg(sp.c1 + jrow) : cz();
  const float2 tap0 = row_ok ? __ldg(sp.tap0 + jrow) : cz();
  const float2 tap1 = row_ok ? __ldg(sp.tap1 + jrow) : cz();
  const bool has_acc = p.acc != nullptr;
  // z before the tile, for the even lane's first sample of chunk 0
  const float2 zb = (row_ok && !odd && tfirst > 0) ? __ldg(sp.zin + jrow * p.N + n0 - 1) : cz();

  // this tile's 16 saved entry slots of each row (one per 8 samples)
  float4 *gst = stage;                                    // g staging, 16 rows x 128 B
  float4 *dst = stage + 128;                              // grad_z staging
  const float2 *ent = reinterpret_cast<const float2 *>(stage + 256);  // [16 rows][16 slots], swizzled
  {
    const long long jt = tfirst / kFbtTile;
    const int s0 = (int)(tfirst - jt * kFbtTile) / kFbtK;
    float4 *ent4 = stage + 256;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int e4 = it * 32 + lane;
      const int rr = e4 >> 3, k = e4 & 7;
      const long long jj = jw0 + rr;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (jj < p.M)
        v = __ldg(reinterpret_cast<const float4 *>(
            sp.carries + fbt_slot(jj * sp.batch + bidx, sp.fbt_ntiles, (int)jt) + s0 + 2 * k));
      ent4[rr * 8 + (k ^ (rr & 7))] = v;
    }
    __syncwarp();
  }

  float2 D = cz();  // d at the sample after the chunk
  if (step > 0) {
    const long long pred = (tile - sp.chains) * 2 + rank;
    const bool ok = scan_link_wait(sp.flags + pred * 4 + quarter, abort_word, abort);
    if (!__all_sync(0xffffffffu, ok)) return false;
    const float4 l = __ldcg(sp.link + pred * 64 + quarter * 16 + r_own);
    D = make_float2(l.x, l.y);
  }
  const float2 mu = c_conj(lam);
  const float2 T0X = make_float2(tap0.x, tap0.x), T0Y = make_float2(tap0.y, -tap0.y);
  const float2 T1X = make_float2(tap1.x, tap1.x), T1Y = make_float2(tap1.y, -tap1.y);
  float2 pc1 = cz(), qc1 = cz(), pt0 = cz(), qt0 = cz(), pt1 = cz(), qt1 = cz();
  const int own = r_own * 8, sw = r_own & 7, half = odd ? 4 : 0;
  // the ring's loads two chunks ahead: chunks c - 2 of this tile, then the
  // first two of the warp's next tile
  int xn = 0, yn = 0;
  const bool has_next =
      lane == 0 && ring_coords(tile + ring.npairs, kBN / 32 - 1, p, sp, rank, quarter, xn, yn);

#pragma unroll 1
  for (int c = kBN / 32 - 1; c >= 0; --c) {
    const long long nbase = n0 + c * 16;
    const uint32_t kseq = ring.consumed;
    bool ok = mbar_wait(ring.bar + (kseq & 1), (kseq >> 1) & 1u, abort, 8);
    // chunk c - 1 (the next in the ring) holds the z before the even lane's
    // first sample
    if (c > 0) ok = ok && mbar_wait(ring.bar + ((kseq + 1) & 1), ((kseq + 1) >> 1) & 1u, abort, 8);
    if (!__all_sync(0xffffffffu, ok)) return false;
    const float4 *zs = reinterpret_cast<const float4 *>(ring.base + (kseq & 1) * kRingSlotBytes);
    float2 z[8];
    float4 ac[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 v = zs[own + ((half + q) ^ sw)];
      z[2 * q] = make_float2(v.x, v.y);
      z[2 * q + 1] = make_float2(v.z, v.w);
      ac[q] = has_acc ? zs[128 + own + ((half + q) ^ sw)] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float2 zpe = zb;
    if (c > 0) {
      const float4 q = reinterpret_cast<const float4 *>(
          ring.base + ((kseq + 1) & 1) * kRingSlotBytes)[own + (7 ^ sw)];
      zpe = make_float2(q.z, q.w);
    }

    float v[32];
    tc_ld_32x32b_x32(tbase + (uint32_t)(c * 32), v);
    float r[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) r[i] = __shfl_xor_sync(0xffffffffu, odd ? v[i] : v[16 + i], 1);
    float2 g[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float pr_re = odd ? r[2 * t] : v[2 * t];
      const float pr_im = odd ? r[2 * t + 1] : v[2 * t + 1];
      const float pi_re = odd ? v[16 + 2 * t] : r[2 * t];
      const float pi_im = odd ? v[16 + 2 * t + 1] : r[2 * t + 1];
      const float4 a = ac[t >> 1];
      g[t] = make_float2(pr_re - pi_im + ((t & 1) ? a.z : a.x),
                         pr_im + pi_re + ((t & 1) ? a.w : a.y));
    }
    if (lane == 0) bulk_wait_read<1>();  // the previous g store has read its staging
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q)
      gst[own + ((half + q) ^ sw)] =
          make_float4(g[2 * q].x, g[2 * q].y, g[2 * q + 1].x, g[2 * q + 1].y);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (warp_ok) tma_store_2d(&sp.tmZ, gst, (int)(2 * nbase), (int)jw0);
      bulk_commit();
    }

    // z before each lane's first sample: the even lane's last (odd lane), or
    // the one loaded a chunk ahead (even lane)
    const float2 zx = shfl_xor2(z[7], 1);
    const float2 zp = odd ? zx : zpe;
    float2 bd[8];
    fbt_drive<8>(tap0, tap1, z, zp, bd);
    float2 e = ent[r_own * 16 + ((c ^ sw) << 1) + (odd ? 1 : 0)];
    float2 yp[8], em[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      yp[k] = e;
      e = c_fma(lam, e, bd[k]);
      em[k] = sp.fuse_act ? c_relu_mask(g[k], e) : g[k];
    }
    // the odd lane's fold from D is d at its first sample: the even lane's D
    float2 h = D;
#pragma unroll
    for (int k = 7; k >= 0; --k) h = c_fma(mu, h, em[k]);
    const float2 hx = shfl_xor2(h, 1);
    float2 dn = odd ? D : hx;
    float2 dsw = make_float2(dn.y, dn.x);
    float2 gz[8];
#pragma unroll
    for (int k = 7; k >= 0; --k) {
      const float2 d = c_fma(mu, dn, em[k]);
      const float2 ds = make_float2(d.y, d.x);
      gz[k] = __ffma2_rn(T0X, d, __ffma2_rn(T0Y, ds, __ffma2_rn(T1X, dn, __fmul2_rn(T1Y, dsw))));
      const float2 dx = make_float2(d.x, d.x), dy = make_float2(d.y, d.y);
      pc1 = __ffma2_rn(yp[k], dx, pc1);
      qc1 = __ffma2_rn(yp[k], dy, qc1);
      pt0 = __ffma2_rn(z[k], dx, pt0);
      qt0 = __ffma2_rn(z[k], dy, qt0);
      const float2 zk1 = k > 0 ? z[k - 1] : zp;
      pt1 = __ffma2_rn(zk1, dx, pt1);
      qt1 = __ffma2_rn(zk1, dy, qt1);
      dn = d;
      dsw = ds;
    }
    // d at the chunk's first sample (the even lane's) enters the chunk before
    const float2 dx2 = shfl_xor2(dn, 1);
    D = odd ? dx2 : dn;

    if (lane == 0) bulk_wait_read<1>();  // the previous grad_z store has read its staging
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q)
      dst[own + ((half + q) ^ sw)] =
          make_float4(gz[2 * q].x, gz[2 * q].y, gz[2 * q + 1].x, gz[2 * q + 1].y);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (warp_ok) tma_store_2d(&sp.tmAct, dst, (int)(2 * nbase), (int)jw0);
      bulk_commit();
      // every lane has used slot kseq: its next chunk
      if (c >= 2)
        ring_issue(ring, kseq + 2, p, sp, (int)(2 * (n0 + 16 * (c - 2))), (int)jw0);
      else if (has_next)
        ring_issue(ring, kseq + 2, p, sp, xn - 32 * (1 - c), yn);
    }
    ring.consumed = kseq + 1;
  }

  // the tile's sums per row: conj(v) d = (v.x d.x + v.y d.y, v.x d.y - v.y d.x)
  {
    float2 s1 = make_float2(pc1.x + qc1.y, qc1.x - pc1.y);
    float2 s2 = make_float2(pt0.x + qt0.y, qt0.x - pt0.y);
    float2 s3 = make_float2(pt1.x + qt1.y, qt1.x - pt1.y);
    s1 = c_add(s1, shfl_xor2(s1, 1));
    s2 = c_add(s2, shfl_xor2(s2, 1));
    s3 = c_add(s3, shfl_xor2(s3, 1));
    if (!odd && row_ok) {
      float2 *pp = sp.partials + ((jrow * sp.batch + bidx) * sp.tiles_per_row + pos) * 3;
      pp[0] = s1;
      pp[1] = s2;
      pp[2] = s3;
    }
  }
  __syncwarp();  // entry-slot reads done before the next tile overwrites them

  // publish d at the tile's first sample for the tile before it in time
  if (pos > 0) {
    const long long me = tile * 2 + rank;
    if (odd) sp.link[me * 64 + quarter * 16 + r_own] = make_float4(D.x, D.y, 0.f, 0.f);
    __threadfence();
    __syncwarp();
    if (lane == 0) st_release_u32(sp.flags + me * 4 + quarter, 1u);
  }
  return true;
}

template <bool kRealOut, int kScan = 0>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
proj_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmX,
            const Params p, const __grid_constant__ ScanParams sp) {
  static_assert(!(kRealOut && kScan), "the scan epilogue runs on the complex output");
  using L = ProjLayout<kRealOut, kScan>;
  constexpr int kStages = L::kStages;
  constexpr int kStageBytes = L::kStageBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  uint64_t *full = bars;                 // this CTA's TMA landed  (1 arrival + tx)
  uint64_t *ready = bars + kStages;      // X' split done, both CTAs (leader's; 8 warps)
  uint64_t *empty = bars + 2 * kStages;  // MMAs done with stage  (leader's commit)
  uint64_t *accf = bars + 3 * kStages;   // accumulator complete  (leader's commit)
  uint64_t *acce = accf + kAccBufs;      // accumulator drained, both CTAs (leader's; 8 warps)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acce + kAccBufs);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
  uint64_t *ringbar = reinterpret_cast<uint64_t *>(tmem_slot + 2);  // backward scan: 4 warps x 2

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = pair_rank();
  const long long pair0 = pair_index(), npairs = pair_count();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 8);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < kAccBufs; ++a) {
      mbar_init(&accf[a], 1);
      mbar_init(&acce[a], 8);
    }
    if constexpr (kScan == kScanBwd)
      for (int i = 0; i < 8; ++i) mbar_init(&ringbar[i], 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmX);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tc_fence_before();
  }
  __syncthreads();
  pair_sync();  // both CTAs' barriers initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (long long tile = pair0; ok && tile < p.num_tiles; tile += npairs) {
        int mp, nt;
        tile_coords(tile, p, mp, nt, kScan ? &sp : nullptr);
        const int arow = mp * kPairM + (int)rank * kBM;
        const int xcol = nt * kBN + (int)rank * kBNh;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort, 1)) {
            ok = false;
            break;
          }
          uint8_t *st = smem + stage * kStageBytes;
          mbar_expect_tx(&full[stage], kTxBytes);
          tma_load_2d(st, &tmA, &full[stage], kb * kBK, arow);
          tma_load_2d(st + kABytes, &tmA, &full[stage], kb * kBK, p.a_rows_pad + arow);
          if (kRealOut) {  // samples [xcol, xcol + 128) of complex rows [8 kb, 8 kb + 8)
            tma_load_2d(st + kRawXOff, &tmX, &full[stage], 2 * xcol, kb * (kBK / 2));
          } else {
#pragma unroll
            for (int i = 0; i < kNBlocks; ++i)
              tma_load_2d(st + 2 * kABytes + i * (kBK * 128), &tmX, &full[stage], xcol + i * 32,
                          kb * kBK);
          }
          ++issued;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Wait for the copies still in flight (the last min(issued, kStages)).
      for (int i = 0; i < kStages && i < issued; ++i) {
        if (--stage < 0) {
          stage = kStages - 1;
          phase ^= 1u;
        }
        mbar_drain(&full[stage], phase);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer (leader)
    if (rank == 0 && lane == 0) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      uint64_t *last = nullptr;
      uint32_t last_parity = 0;
      for (long long tile = pair0; ok && tile < p.num_tiles; tile += npairs) {
        if (!mbar_wait(&acce[acc], acc_phase ^ 1u, abort, 3)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kBN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&ready[stage], phase, abort, 4)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + stage * kStageBytes);
          // A': K-major 64-byte rows, 8-row groups 512 B apart.  X': MN-major,
          // 32-column (128-byte) blocks kBK*128 B apart (LBO), 4-row groups
          // 512 B apart (SBO).  Both CTAs hold their halves at these offsets.
          const uint64_t a_hi = smem_desc(st, 16, 512, kSwizzle64B);
          const uint64_t a_lo = smem_desc(st + kABytes, 16, 512, kSwizzle64B);
          const uint64_t b_hi = smem_desc(st + 2 * kABytes, kBK * 128, 512, kSwizzle128BBase32);
          const uint64_t b_lo =
              smem_desc(st + 2 * kABytes + kBBytes, kBK * 128, 512, kSwizzle128BBase32);
#pragma unroll
          for (int ks = 0; ks < kBK / kUmmaK; ++ks) {
            // A advances 32 bytes along K inside its 64-byte swizzle row; X'
            // advances 8 rows (1024 bytes) per K step.
            const uint64_t da = (uint64_t)(ks * (kUmmaK * 4) >> 4);
            const uint64_t db = (uint64_t)(ks * (kUmmaK * 128) >> 4);
            const uint32_t accum = (kb > 0 || ks > 0) ? 1u : 0u;
            tc_mma_pair_tf32(d_tmem, a_hi + da, b_hi + db, kIdesc, accum);
            tc_mma_pair_tf32(d_tmem, a_hi + da, b_lo + db, kIdesc, 1u);
            tc_mma_pair_tf32(d_tmem, a_lo + da, b_hi + db, kIdesc, 1u);
          }
          tc_commit_pair(cluster_addr(&empty[stage], 0));
          tc_commit_pair(cluster_addr(&empty[stage], 1));
          last = &empty[stage];
          last_parity = phase;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair(cluster_addr(&accf[acc], 0));
        tc_commit_pair(cluster_addr(&accf[acc], 1));
        if (++acc == kAccBufs) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // The MMAs read both CTAs' shared memory and write both TMEMs
      // asynchronously: the last commit must land before either CTA frees them.
      if (last != nullptr) mbar_drain(last, last_parity);
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------- epilogue
    const int quarter = warp & 3;          // TMEM lanes this warp may read
    const int row = quarter * 32 + lane;   // A' row within this CTA's half of the tile
    const bool odd = (row & 1) != 0;
    const uint32_t acce0 = cluster_addr(&acce[0], 0);
    const uint32_t acce1 = cluster_addr(&acce[1], 0);
    float4 *stage =
        reinterpret_cast<float4 *>(smem + L::kStagingOff + quarter * L::kWarpStaging);
    int acc = 0;
    uint32_t acc_phase = 0;
    if constexpr (kScan == kScanFwd) {  // every thread's entry is saved (the row kernels' marker)
      if (blockIdx.x == 0 && warp == 2 && lane == 0)
        sp.carries[fbt_marker(p.M * sp.batch, sp.fbt_ntiles)] = make_float2(1.f, 0.f);
    }
    ScanRing ring{smem + L::kRingOff + quarter * kRingWarpBytes, ringbar + 2 * quarter, npairs,
                  0u, 0u};
    if constexpr (kScan == kScanBwd) {  // the first two chunks of this warp's sequence
      int x0, y0;
      if (lane == 0 && ring_coords(pair0, kBN / 32 - 1, p, sp, (int)rank, quarter, x0, y0)) {
        prefetch_tmap(&sp.tmZin);
        if (p.acc) prefetch_tmap(&sp.tmAcc);
        ring_issue(ring, 0, p, sp, x0, y0);
        ring_issue(ring, 1, p, sp, x0 - 32, y0);
      }
    }
    for (long long tile = pair0; tile < p.num_tiles; tile += npairs) {
      // every lane waits; the decision is made warp-uniform before the
      // .sync.aligned TMEM loads
      const bool ok = mbar_wait(&accf[acc], acc_phase, abort, 5);
      if (!__all_sync(0xffffffffu, ok)) {
        if (kScan && lane == 0) st_relaxed_u32(sp.flags + p.num_tiles * 8, 1u);
        break;
      }
      tc_fence_after();
      int mp, nt;
      tile_coords(tile, p, mp, nt, kScan ? &sp : nullptr);
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * kBN);
      // Each chunk of 32 TMEM columns gives this warp 16 output rows x W
      // samples (W = 16 complex X, 32 real X).  The lanes combine their
      // products into complex outputs, stage them in shared memory (16-byte
      // chunk k of row r at k ^ (r & 7): conflict-free both ways), and write
      // them back as whole rows, 8 or 16 lanes per row, so every store
      // instruction covers full 128-byte lines (and so does the acc load).
      if (kRealOut) {
        // lane = output row jr; each chunk is 32 consecutive samples of it,
        // staged (chunk k of row r at k ^ (r & 7)) and written as whole
        // 128-byte row pieces, 8 lanes per row
        const long long jr0 = (long long)mp * kPairM + (long long)rank * kBM + quarter * 32;
#pragma unroll 1
        for (int c = 0; c < kBN / 32; ++c) {
          float v[32];
          tc_ld_32x32b_x32(tbase + (uint32_t)(c * 32), v);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            stage[lane * 8 + (k ^ (lane & 7))] =
                make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
          __syncwarp();
          const long long nbase = (long long)nt * kBN + c * 32;
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int e = it * 32 + lane;
            const int rr = e >> 3, k = e & 7;
            const long long jj = jr0 + rr, n = nbase + 4 * k;  // N % 4 == 0
            if (jj < p.M && n < p.N)
              *reinterpret_cast<float4 *>(p.out_real + jj * p.N + n) = stage[rr * 8 + (k ^ (rr & 7))];
          }
          __syncwarp();
        }
      } else if constexpr (kScan == kScanFwd) {
        if (!scan_epilogue(tbase, stage, p, sp, tile, mp, nt, rank, quarter, lane, abort)) break;
      } else if constexpr (kScan == kScanBwd) {
        if (!scan_bwd_epilogue(tbase, stage, p, sp, tile, mp, nt, rank, quarter, lane, ring,
                               abort))
          break;
      } else {
      const int W = p.real_x ? 32 : 16;            // samples per row per chunk
      const int kpr = W / 2;                       // 16-byte chunks per row
      const long long jw0 = ((long long)mp * kPairM + (long long)rank * kBM + quarter * 32) >> 1;
      const int r_own = lane >> 1;
      const int iters = 16 * kpr / 32;             // 16-byte pieces per lane per chunk
      if (p.acc != nullptr && lane < 16) {
        // Into L2: this warp's 16 rows of acc for its next tile (and, on the
        // pair's first tile, for this one), so that the chunk loads below hit
        // L2 instead of waiting on HBM.
        const int bytes = (p.real_x ? kBN : kBN / 2) * 8;
        for (int ahead = (tile < npairs) ? 0 : 1; ahead < 2; ++ahead) {
          const long long t2 = tile + ahead * npairs;
          if (t2 >= p.num_tiles) break;
          int mp2, nt2;
          tile_coords(t2, p, mp2, nt2);
          const long long j2 =
              (((long long)mp2 * kPairM + (long long)rank * kBM + quarter * 32) >> 1) + lane;
          const long long n2 = p.real_x ? (long long)nt2 * kBN : (long long)nt2 * (kBN / 2);
          if (j2 < p.M && n2 < p.N) {
            const long long left = (p.N - n2) * 8;
            const int nb = (int)(left < bytes ? left : bytes);  // N is even: a multiple of 16
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p.acc + j2 * p.N + n2),
                         "r"(nb)
                         : "memory");
          }
        }
      }
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        const long long nbase = p.real_x ? (long long)nt * kBN + c * 32
                                         : (long long)nt * (kBN / 2) + c * 16;
        // this lane's acc pieces, loaded first so that their latency hides
        // behind the TMEM load and the staging
        float4 av[8];
        if (p.acc) {
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            av[it] = make_float4(0.f, 0.f, 0.f, 0.f);
            const int e = it * 32 + lane;
            const int rr = e / kpr, k = e - rr * kpr;
            const long long jj = jw0 + rr, n = nbase + 2 * k;
            if (it < iters && jj < p.M && n < p.N)
              av[it] = *reinterpret_cast<const float4 *>(p.acc + jj * p.N + n);
          }
        }
        float v[32];
        tc_ld_32x32b_x32(tbase + (uint32_t)(c * 32), v);
        float r[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) r[i] = __shfl_xor_sync(0xffffffffu, odd ? v[i] : v[16 + i], 1);
        if (p.real_x) {
          // lane 2j holds Re, lane 2j+1 Im of samples 0..31: the even lane
          // keeps samples 0..15, the odd lane 16..31
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 o = odd ? make_float4(r[2 * q], v[16 + 2 * q], r[2 * q + 1], v[17 + 2 * q])
                                 : make_float4(v[2 * q], r[2 * q], v[2 * q + 1], r[2 * q + 1]);
            const int k = (odd ? 8 : 0) + q;
            stage[r_own * kpr + (k ^ (r_own & 7))] = o;
          }
        } else {
          // complex X: P[2j, 2n], P[2j+1, 2n+1] etc. give out[j, n]; the even
          // lane keeps samples 0..7, the odd lane 8..15
          float2 z[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const float pr_re = odd ? r[2 * t] : v[2 * t];
            const float pr_im = odd ? r[2 * t + 1] : v[2 * t + 1];
            const float pi_re = odd ? v[16 + 2 * t] : r[2 * t];
            const float pi_im = odd ? v[16 + 2 * t + 1] : r[2 * t + 1];
            z[t] = make_float2(pr_re - pi_im, pr_im + pi_re);
          }
          if (p.inplace) {
            // two 2 KB halves in turn; a half is reused once the reduce that
            // read it two chunks ago has finished reading
            float4 *st2 = stage + (c & 1) * 128;
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int k = (odd ? 4 : 0) + q;
              st2[r_own * 8 + (k ^ (r_own & 7))] =
                  make_float4(z[2 * q].x, z[2 * q].y, z[2 * q + 1].x, z[2 * q + 1].y);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              // a box wholly past N is skipped; a partial one is clipped by the map
              if (jw0 < p.M && nbase < p.N) tma_reduce_add_2d(&sp.tmZ, st2, (int)(2 * nbase), (int)jw0);
              bulk_commit();
            }
            continue;
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int k = (odd ? 4 : 0) + q;
            stage[r_own * kpr + (k ^ (r_own & 7))] =
                make_float4(z[2 * q].x, z[2 * q].y, z[2 * q + 1].x, z[2 * q + 1].y);
          }
        }
        __syncwarp();
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          if (it < iters) {
            const int e = it * 32 + lane;
            const int rr = e / kpr, k = e - rr * kpr;
            float4 o = stage[rr * kpr + (k ^ (rr & 7))];
            const long long jj = jw0 + rr;
            const long long n = nbase + 2 * k;  // even; N is even, so n < N covers n + 1
            if (jj < p.M && n < p.N) {
              if (p.acc) o = make_float4(o.x + av[it].x, o.y + av[it].y, o.z + av[it].z, o.w + av[it].w);
              *reinterpret_cast<float4 *>(p.out + jj * p.N + n) = o;
            }
          }
        }
        __syncwarp();
      }
      }  // complex output
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? acce1 : acce0);
      if (++acc == kAccBufs) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (kScan || p.inplace) {  // the TMA stores of this warp complete before the CTA exits
      if (lane == 0) bulk_wait<0>();
      __syncwarp();
    }
    if constexpr (kScan == kScanBwd) {  // and so do its ring loads (after an abort: bounded)
      if (lane == 0)
        for (uint32_t k = ring.consumed; k < ring.issued; ++k)
          mbar_drain(ring.bar + (k & 1), (k >> 1) & 1u);
      __syncwarp();
    }
  } else {
    // ---------------------------------------------------------- transform
    const int t = threadIdx.x - 6 * 32;  // 0..127
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (long long tile = pair0; ok && tile < p.num_tiles; tile += npairs) {
      for (int kb = 0; kb < p.k_blocks; ++kb) {
        ok = __all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort, 2));
        if (!ok) break;
        float4 *xb = reinterpret_cast<float4 *>(smem + stage * kStageBytes + 2 * kABytes);
        float4 *xl = reinterpret_cast<float4 *>(smem + stage * kStageBytes + 2 * kABytes + kBBytes);
        if (kRealOut) {
          // raw row k (complex k index 8 kb + k): 128 samples as (Re, Im); B
          // row k takes the Re plane, row 8 + k the Im plane, 4 samples per
          // item (16 bytes inside one 32-byte atom of the MN-major layout)
          const uint8_t *raw = smem + stage * kStageBytes + kRawXOff;
          uint8_t *bh = reinterpret_cast<uint8_t *>(xb), *bl = reinterpret_cast<uint8_t *>(xl);
#pragma unroll
          for (int e = t; e < 8 * (kBNh / 4); e += 128) {
            const int k = e / (kBNh / 4), g4 = e - k * (kBNh / 4);
            const float4 a = *reinterpret_cast<const float4 *>(raw + k * (kBNh * 8) + g4 * 32);
            const float4 b = *reinterpret_cast<const float4 *>(raw + k * (kBNh * 8) + g4 * 32 + 16);
            const float4 re = make_float4(a.x, a.z, b.x, b.z), im = make_float4(a.y, a.w, b.y, b.w);
            const uint32_t ore = mn32_offset(4 * g4, k), oim = mn32_offset(4 * g4, k + 8);
            *reinterpret_cast<float4 *>(bh + ore) = re;
            *reinterpret_cast<float4 *>(bh + oim) = im;
            *reinterpret_cast<float4 *>(bl + ore) = make_float4(tf32_lo(re.x), tf32_lo(re.y), tf32_lo(re.z), tf32_lo(re.w));
            *reinterpret_cast<float4 *>(bl + oim) = make_float4(tf32_lo(im.x), tf32_lo(im.y), tf32_lo(im.z), tf32_lo(im.w));
          }
        } else {
#pragma unroll
          for (int i = t; i < kBBytes / 16; i += 128) {
            const float4 v = xb[i];  // stays in place as the hi part
            xl[i] = make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
          }
        }
        // generic-proxy smem writes -> visible to the tensor core (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(cluster_addr(&ready[stage], 0));
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  }

  __syncwarp();  // lanes of warps 0 and 1 wait for their elected lane's loop
  tc_fence_before();
  __syncthreads();
  pair_sync();  // no MMA, commit or remote arrival of either CTA is still pending
  if (warp == 1) {
    tc_fence_after();
    tmem_free_pair(tmem_base, kTmemCols);
  }
}


// ------------------------------------------------------------ weight gradient
// gW[j, i] = sum_n gz[j, n] conj(h[i, n]): the weight cotangent of z = W h.
// Over the interleaved samples k' = 2n + {0: Re, 1: Im},
//   Re gW[j,i] = sum_k' gz'[j,k'] h'[i,k'],    Im gW[j,i] = sum_k' gz'[j,k'] h~'[i,k'],
// with h~'[i,2n] = -Im h[i,n] and h~'[i,2n+1] = Re h[i,n].  A CTA pair owns a
// work tile of 256 j x 128 i: A = gz' (each CTA 128 j rows), B = 256 columns,
// CTA r's half being [h' ; h~'] of the 64 rows i0 + 64r + [0, 64).  Both
// operands are K-major, as TMA lands them (128-byte swizzle): h' is its own hi
// part, and h~' is a swap-and-negate of each (Re, Im) pair inside a 16-byte
// chunk, so the transform warps only rewrite chunks in place order (lo parts
// and h~'), with no transpose.  Each CTA's TMEM holds D[j][c] for its 128 j:
// column c = 128h + 64q + e holds (q = 0: Re, 1: Im) gW[j, i0 + 64h + e].  The
// k' range is split over CTA pairs (split-K); each CTA stores its fp32
// partial tile and proj_wgrad_reduce_kernel sums the partials in a fixed
// order (deterministic).
//
// Stage (64 KB per CTA, 32 k' per row): A_hi = gz' (TMA, 16 KB) | B_hi = h'
// (TMA, 8 KB), h~' (8 KB) | A_lo (16 KB) | B_lo = h'_lo, h~'_lo (16 KB).
constexpr int kWgRows = 128;                     // j rows per CTA
constexpr int kWgPairRows = 2 * kWgRows;         // j rows per pair tile
constexpr int kWgCols = 128;                     // i per pair tile
constexpr int kWgHRows = kWgCols / 2;            // h' rows each CTA stages
// Real gz (the readout's cotangent): a stage also holds the raw h' tile, 64
// rows x 16 samples x (Re, Im) = 128-byte rows (128-byte swizzle), which the
// transform de-interleaves into the Re and -Im planes of B.
//
// Both forms stage 32 k per row (128-byte rows, 128-byte swizzle): every row
// the tile touches is a separate piece of gz or h (rows are N samples apart,
// 4 MB at the config-5 layer), and a k-block touches 192 such rows per CTA;
// 128-byte pieces halve the row accesses per byte against 64-byte ones (1.33
// -> 1.09 ms for the complex form at the config-5 layer).  Real gz lands its
// raw h tile (64 rows x 32 samples x (Re, Im), two 128-byte boxes) in the
// B_lo region, which the transform overwrites row by row after reading it.
template <bool kRealGz>
struct WgLayout {
  static constexpr int kBKw = 2 * kBK;                       // k (k' or samples) per stage
  static constexpr int kABytes = kWgRows * kBKw * 4;         // 16 KB
  static constexpr int kHBytes = kWgHRows * kBKw * 4;        // 8 KB
  static constexpr int kRawOff = 2 * kABytes + 2 * kHBytes;  // 48 KB: the B_lo region
  static constexpr int kStages = 3;
  static constexpr int kStageBytes = 2 * kABytes + 4 * kHBytes;  // 64 KB
  static constexpr int kTxBytes = kRealGz ? kABytes + 2 * kHBytes : kABytes + kHBytes;
  static constexpr uint64_t kSwz = 2;                        // 128-byte swizzle
  static constexpr uint32_t kSbo = 1024;                     // 8 rows of 128 bytes
  static constexpr int kChunk = 8;                           // k-blocks per fold: 96 MMAs
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarBytes + kStagingBytes + 1024;
};
// TMEM: columns [0, 256) the CTA's running total, [256, 512) the chunk
// accumulator.  The tensor core's fp32 accumulate rounds with a bias that
// grows with the number of accumulations into one accumulator (about 2e-4
// relative after 10^4 of them, against ~5e-6 after 10^2), so the MMAs
// accumulate WgLayout::kChunk k-blocks (96 MMAs) at a time and the epilogue
// warps fold each chunk into the total with ordinary fp32 adds.
constexpr int kWgTmemCols = 2 * kBN;

struct WgParams {
  float2 *partials;          // [splits][m_pairs*256][ld] complex
  long long M, K;            // gW is M x K (F_out x F_in)
  int m_pairs, i_tiles, splits;
  long long kblocks;         // ceil(2N / kBK)
  int ld;                    // i_tiles * 128
};

// 10 warps: 0 TMA, 1 MMA (leader) / TMEM, 2..5 epilogue, 6..9 transform.
constexpr int kWgThreads = 320;

__device__ __forceinline__ float4 swap_neg(float4 v) { return make_float4(-v.y, v.x, -v.w, v.z); }
__device__ __forceinline__ float4 tf32_lo4(float4 v) {
  return make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
}

// kRealGz: gz is real (M x N) and the reduction runs over the N samples:
// Re gW = sum_n gz h_re, Im gW = sum_n gz (-h_im); A = gz as TMA lands it,
// B = the de-interleaved [h_re ; -h_im] rows.  Half the k-blocks of the
// complex form, whose A would be gz interleaved with zeros.
template <bool kRealGz>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kWgThreads, 1)
proj_wgrad_kernel(const __grid_constant__ CUtensorMap tmG, const __grid_constant__ CUtensorMap tmH,
                  const WgParams p) {
  using L = WgLayout<kRealGz>;
  constexpr int kWgStages = L::kStages;
  constexpr int kWgStageBytes = L::kStageBytes;
  constexpr int kWgTxBytes = L::kTxBytes;
  constexpr int kWgABytes = L::kABytes;
  constexpr int kWgHBytes = L::kHBytes;
  constexpr int kWgRawOff = L::kRawOff;
  constexpr int kWgChunk = L::kChunk;
  constexpr int kBKw = L::kBKw;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kWgStages * kWgStageBytes);
  uint64_t *full = bars;                   // this CTA's TMA landed   (1 + tx)
  uint64_t *ready = full + kWgStages;      // operands written, both CTAs (leader's; 8 warps)
  uint64_t *empty = ready + kWgStages;     // MMAs done with stage   (leader's commit)
  uint64_t *accf = empty + kWgStages;      // chunk accumulated      (leader's commit)
  uint64_t *acce = accf + 1;               // chunk folded, both CTAs (leader's; 8 warps)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acce + 1);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = pair_rank();
  // tile fastest: the pairs that share a gz' or h' block over the same k
  // range are neighbours in launch order and progress together, so the block
  // is read from HBM once and from L2 by its second user
  const int ntiles = p.m_pairs * p.i_tiles;
  const int pid = (int)pair_index();
  const int split = pid / ntiles;
  const int tile = pid - split * ntiles;
  const int mp = tile % p.m_pairs;
  const int it = tile / p.m_pairs;
  const long long kb0 = (long long)split * p.kblocks / p.splits;
  const long long kb1 = (long long)(split + 1) * p.kblocks / p.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWgStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 8);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    mbar_init(acce, 8);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tmG);
    prefetch_tmap(&tmH);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kWgTmemCols);
    tc_fence_before();
  }
  __syncthreads();
  pair_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      const int jrow = mp * kWgPairRows + (int)rank * kWgRows;
      const int irow = it * kWgCols + (int)rank * kWgHRows;
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      for (long long kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort, 1)) break;
        uint8_t *st = smem + stage * kWgStageBytes;
        mbar_expect_tx(&full[stage], kWgTxBytes);
        tma_load_2d(st, &tmG, &full[stage], (int)(kb * kBKw), jrow);
        if (kRealGz) {  // h' floats [64 kb, 64 kb + 64): samples [32 kb, 32 kb + 32)
          tma_load_2d(st + kWgRawOff, &tmH, &full[stage], (int)(kb * 2 * kBKw), irow);
          tma_load_2d(st + kWgRawOff + kWgHBytes, &tmH, &full[stage], (int)(kb * 2 * kBKw + kBKw),
                      irow);
        } else
          tma_load_2d(st + kWgABytes, &tmH, &full[stage], (int)(kb * kBKw), irow);
        ++issued;
        if (++stage == kWgStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      for (int i = 0; i < kWgStages && i < issued; ++i) {
        if (--stage < 0) {
          stage = kWgStages - 1;
          phase ^= 1u;
        }
        mbar_drain(&full[stage], phase);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer (leader)
    if (rank == 0 && lane == 0) {
      int stage = 0;
      uint32_t phase = 0, cphase = 0;
      bool ok = true;
      uint64_t *last = nullptr;
      uint32_t last_parity = 0;
      const uint32_t d_tmem = tmem_base + (uint32_t)kBN;  // chunk accumulator
      for (long long c0 = kb0; ok && c0 < kb1; c0 += kWgChunk) {
        const long long c1 = c0 + kWgChunk < kb1 ? c0 + kWgChunk : kb1;
        if (!mbar_wait(acce, cphase ^ 1u, abort, 3)) break;  // previous chunk read out
        tc_fence_after();
        for (long long kb = c0; kb < c1; ++kb) {
          if (!mbar_wait(&ready[stage], phase, abort, 4)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + stage * kWgStageBytes);
          const uint64_t a_hi = smem_desc(st, 16, L::kSbo, L::kSwz);
          const uint64_t b_hi = smem_desc(st + kWgABytes, 16, L::kSbo, L::kSwz);
          const uint64_t a_lo = smem_desc(st + kWgABytes + 2 * kWgHBytes, 16, L::kSbo, L::kSwz);
          const uint64_t b_lo =
              smem_desc(st + 2 * kWgABytes + 2 * kWgHBytes, 16, L::kSbo, L::kSwz);
#pragma unroll
          for (int ks = 0; ks < kBKw / kUmmaK; ++ks) {
            const uint64_t dk = (uint64_t)(ks * (kUmmaK * 4) >> 4);  // 32 B along K
            const uint32_t accum = (kb > c0 || ks > 0) ? 1u : 0u;
            tc_mma_pair_tf32(d_tmem, a_hi + dk, b_hi + dk, kIdescKK, accum);
            tc_mma_pair_tf32(d_tmem, a_hi + dk, b_lo + dk, kIdescKK, 1u);
            tc_mma_pair_tf32(d_tmem, a_lo + dk, b_hi + dk, kIdescKK, 1u);
          }
          tc_commit_pair(cluster_addr(&empty[stage], 0));
          tc_commit_pair(cluster_addr(&empty[stage], 1));
          last = &empty[stage];
          last_parity = phase;
          if (++stage == kWgStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair(cluster_addr(accf, 0));
        tc_commit_pair(cluster_addr(accf, 1));
        last = accf;
        last_parity = cphase;
        cphase ^= 1u;
      }
      if (last != nullptr) mbar_drain(last, last_parity);
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const uint32_t acce_leader = cluster_addr(acce, 0);
    float4 *stage = reinterpret_cast<float4 *>(smem + kWgStages * kWgStageBytes + kBarBytes +
                                               quarter * (kStagingBytes / 4));
    const long long nchunks = (kb1 - kb0 + kWgChunk - 1) / kWgChunk;
    uint32_t cphase = 0;
    bool ok = true;
    for (long long q = 0; q < nchunks; ++q) {
      ok = __all_sync(0xffffffffu, mbar_wait(accf, cphase, abort, 5));
      if (!ok) break;
      tc_fence_after();
      if (q + 1 < nchunks) {
        // total += chunk (the first chunk initialises the total)
#pragma unroll 1
        for (int c = 0; c < kBN / 32; ++c) {
          float v[32];
          tc_ld_32x32b_x32(tbase + (uint32_t)(kBN + c * 32), v);
          if (q > 0) {
            float t[32];
            tc_ld_32x32b_x32(tbase + (uint32_t)(c * 32), t);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] += t[i];
          }
          tc_st_32x32b_x32(tbase + (uint32_t)(c * 32), v);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      } else {
        // last chunk: partial = total + chunk; columns 128h + 64q + e hold
        // (q = 0: Re, 1: Im) of i = i0 + 64h + e.  16 outputs of each of the
        // warp's 32 rows at a time go through shared memory (chunk k of row
        // r at k ^ (r & 7)) and out as whole 128-byte row pieces.
        const long long jrow0 =
            (long long)mp * kWgPairRows + (long long)rank * kWgRows + quarter * 32;
        float2 *dst0 = p.partials + ((long long)split * p.m_pairs * kWgPairRows + jrow0) * p.ld +
                       (long long)it * kWgCols;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          const int col = (c >> 1) * 128 + (c & 1) * 32;  // Re columns; Im at col + 64
          float re[32], im[32];
          tc_ld_32x32b_x32(tbase + (uint32_t)(kBN + col), re);
          tc_ld_32x32b_x32(tbase + (uint32_t)(kBN + col + 64), im);
          if (q > 0) {
            float t[32];
            tc_ld_32x32b_x32(tbase + (uint32_t)col, t);
#pragma unroll
            for (int i = 0; i < 32; ++i) re[i] += t[i];
            tc_ld_32x32b_x32(tbase + (uint32_t)(col + 64), t);
#pragma unroll
            for (int i = 0; i < 32; ++i) im[i] += t[i];
          }
#pragma unroll
          for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int i = half * 16 + 2 * k;
              stage[lane * 8 + (k ^ (lane & 7))] = make_float4(re[i], im[i], re[i + 1], im[i + 1]);
            }
            __syncwarp();
#pragma unroll
            for (int itr = 0; itr < 8; ++itr) {
              const int e = itr * 32 + lane;
              const int rr = e >> 3, k = e & 7;
              *reinterpret_cast<float4 *>(dst0 + (long long)rr * p.ld + c * 32 + half * 16 + 2 * k) =
                  stage[rr * 8 + (k ^ (rr & 7))];
            }
            __syncwarp();
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce_leader);
      cphase ^= 1u;
    }
  } else {
    // ---------------------------------------------------------- transform
    // Chunk-wise (16 bytes = two (Re, Im) pairs): every derived operand sits
    // at the same offset within its region as the TMA chunk it comes from, so
    // the 64-byte swizzle carries over unchanged.
    const int t = threadIdx.x - 6 * 32;  // 0..127
    int stage = 0;
    uint32_t phase = 0;
    for (long long kb = kb0; kb < kb1; ++kb) {
      if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort, 2))) break;
      uint8_t *st = smem + stage * kWgStageBytes;
      const float4 *ah = reinterpret_cast<const float4 *>(st);
      float4 *bh = reinterpret_cast<float4 *>(st + kWgABytes);
      float4 *al = reinterpret_cast<float4 *>(st + kWgABytes + 2 * kWgHBytes);
      float4 *bl = reinterpret_cast<float4 *>(st + 2 * kWgABytes + 2 * kWgHBytes);
      constexpr int kAChunks = kWgABytes / 16, kHChunks = kWgHBytes / 16;
#pragma unroll
      for (int i = t; i < kAChunks; i += 128) al[i] = tf32_lo4(ah[i]);
      if (kRealGz) {
        // One thread per h' row r (t < 64): the raw row is two 128-byte rows
        // (samples 0..15 and 16..31 as (Re, Im) pairs, 16-byte chunk q of row
        // r at q ^ (r & 7)) in the B_lo region.  The thread reads all 16 of
        // its raw chunks first, then writes the Re and -Im planes (chunk c =
        // samples 4c..4c+3 at c ^ (r & 7)) to B_hi and their lo parts over
        // its own raw row, so no thread overwrites bytes another still reads.
        if (t < kWgHRows) {
          const int r = t, sw = r & 7;
          const uint8_t *raw = st + kWgRawOff + r * 128;
          float4 v[16];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            v[q] = *reinterpret_cast<const float4 *>(raw + ((q ^ sw) << 4));
            v[8 + q] = *reinterpret_cast<const float4 *>(raw + kWgHBytes + ((q ^ sw) << 4));
          }
          uint8_t *hre = st + kWgABytes + r * 128, *him = hre + kWgHBytes;
          uint8_t *lre = st + kWgRawOff + r * 128, *lim = lre + kWgHBytes;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 a0 = v[2 * c], a1 = v[2 * c + 1];
            const float4 re = make_float4(a0.x, a0.z, a1.x, a1.z);
            const float4 im = make_float4(-a0.y, -a0.w, -a1.y, -a1.w);
            const int o = (c ^ sw) << 4;
            *reinterpret_cast<float4 *>(hre + o) = re;
            *reinterpret_cast<float4 *>(him + o) = im;
            *reinterpret_cast<float4 *>(lre + o) = tf32_lo4(re);
            *reinterpret_cast<float4 *>(lim + o) = tf32_lo4(im);
          }
        }
      } else {
#pragma unroll
        for (int i = t; i < kHChunks; i += 128) {
          const float4 v = bh[i];
          const float4 lo = tf32_lo4(v);
          bh[kHChunks + i] = swap_neg(v);
          bl[i] = lo;
          bl[kHChunks + i] = swap_neg(lo);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_addr(&ready[stage], 0));
      if (++stage == kWgStages) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  pair_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_free_pair(tmem_base, kWgTmemCols);
  }
}

// gW[j, i] = sum over splits of the partial tiles, in a fixed order: a CTA
// owns 32 consecutive outputs; warp g sums the splits s = g, g + 8, ... in
// ascending order (lane = output, so each load is one coalesced 256-byte
// row piece), then the 8 group sums are added in group order, in double.
constexpr int kWgReduceGroups = 8;
__global__ void __launch_bounds__(32 * kWgReduceGroups)
proj_wgrad_reduce_kernel(const float2 *__restrict__ partials, float2 *__restrict__ gw, long long M,
                         long long K, int splits, long long rows_pad, int ld) {
  const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
  const long long e = blockIdx.x * 32LL + lane;
  const bool valid = e < M * K;
  const long long j = valid ? e / K : 0, i = valid ? e - j * K : 0;
  double re = 0.0, im = 0.0;
  if (valid) {
    for (int s = grp; s < splits; s += kWgReduceGroups) {
      const float2 v = partials[((long long)s * rows_pad + j) * ld + i];
      re += v.x;
      im += v.y;
    }
  }
  __shared__ double2 part[kWgReduceGroups][32];
  part[grp][lane] = make_double2(re, im);
  __syncthreads();
  if (grp == 0 && valid) {
    double sr = 0.0, si = 0.0;
#pragma unroll
    for (int g = 0; g < kWgReduceGroups; ++g) {
      sr += part[g][lane].x;
      si += part[g][lane].y;
    }
    gw[e] = make_float2((float)sr, (float)si);
  }
}

}  // namespace proj
}  // namespace rqf
