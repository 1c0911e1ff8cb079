// C-ABI entry points of librqf_b200.so (declared in include/rqf_b200.h).
//
// The entry points validate sizes and alignment, clear the look-back part of
// the caller's scratch with cudaMemsetAsync, pick the kernel instantiation and
// launch on the caller's stream.  Nothing here allocates device memory.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/rqf_b200.h"
#include "btf_scan.cuh"
#include "btf_stream.cuh"
#include "fbt_rows.cuh"
#include "fbt_rank1.cuh"
#include "fbt_scan.cuh"
#include "coeffs.cuh"
#include "lowrank.cuh"
#include "readout.cuh"
#include "reduce.cuh"
#include "projection.cuh"
#include "selective.cuh"

using namespace rqf;

namespace {

constexpr int kAbiVersion = 1;
constexpr int64_t kMaxTickets = 0x7fffffffLL;

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

struct Scratch {
  size_t flags_off, flags_bytes, partials_off, total;
};

inline Scratch scratch_layout(int64_t rows, int64_t ntiles) {
  Scratch s;
  s.flags_bytes = (size_t)rows * (size_t)ntiles * 2 * sizeof(u64);
  const size_t partial_bytes = (size_t)rows * (size_t)ntiles * 3 * sizeof(float2);
  s.flags_off = 256;  // [0, 256): ticket counter
  s.partials_off = s.flags_off + round256(s.flags_bytes);
  s.total = s.partials_off + round256(partial_bytes);
  return s;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// (B,T,F) tiling.  Sub-tiles of 64 steps; the saved entry states are per
// sub-tile, so each launch picks its own tile length: long tiles amortise a
// tile's fixed costs (ticket, header, look-back round trip), but there should
// still be a tile for every SM.
inline int64_t btf_nsub(int64_t T) { return T <= 0 ? 0 : ceil_div(T, (int64_t)kBtfSub); }
inline int btf_log2_tile(int64_t B, int64_t T, int64_t F, int max_log2) {
  const int64_t groups = B * ceil_div(F, 32), nsub = btf_nsub(T);
  int l = max_log2;
  while (l > 0 && ((1LL << (l - 1)) >= nsub || groups * ceil_div(nsub, 1LL << l) < 148)) --l;
  return l;
}
// Scratch of the (B,T,F) kernels: ticket, look-back flags and partials sized
// for one tile per sub-tile (the most tiles any launch uses), then the c1
// power table (kBtfPowLevels x F).
struct BtfScratch {
  Scratch base;
  size_t pw_off, total;
};
inline BtfScratch btf_scratch_layout(int64_t B, int64_t T, int64_t F) {
  BtfScratch s;
  s.base = scratch_layout(B * F, btf_nsub(T));
  s.pw_off = s.base.total;
  s.total = s.pw_off + round256((size_t)kBtfPowLevels * (size_t)F * sizeof(float2));
  return s;
}

inline int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? RQF_OK : RQF_ERR_LAUNCH;
}

// Resident CTAs of a persistent kernel on the current device (sets its dynamic
// shared-memory limit first).  Returns 0 when the kernel cannot be resident.
template <typename Kern>
int64_t resident_ctas(Kern kernel, int threads, size_t smem) {
  int dev = 0, sms = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) !=
      cudaSuccess)
    return 0;
  return (int64_t)sms * per_sm;
}

// Persistent row-sequential launch when every resident CTA gets at least one
// whole row; returns false (nothing launched) when the look-back tile kernels
// should be used instead.
template <typename Kern>
bool launch_rows(Kern kernel, size_t smem, const FbtArgs &a, cudaStream_t stream) {
  if (a.T > 0x7fffffffLL || a.rows > 0x7fffffffLL) return false;  // 32-bit cursors
  const int64_t g = resident_ctas(kernel, kFbtThreads, smem);
  if (g <= 0 || a.rows < g) return false;
  kernel<<<(unsigned)g, kFbtThreads, smem, stream>>>(a);
  return true;
}

inline int zero_complex(float *p, int64_t n, cudaStream_t s) {
  if (!p || n <= 0) return RQF_OK;
  return cudaMemsetAsync(p, 0, (size_t)n * 2 * sizeof(float), s) == cudaSuccess ? RQF_OK
                                                                               : RQF_ERR_LAUNCH;
}

inline int clear_lookback(void *scratch, const Scratch &lay, cudaStream_t s) {
  return cudaMemsetAsync(scratch, 0, lay.flags_off + lay.flags_bytes, s) == cudaSuccess
             ? RQF_OK
             : RQF_ERR_LAUNCH;
}

template <typename T>
inline T *at(void *base, size_t off) {
  return reinterpret_cast<T *>(static_cast<char *>(base) + off);
}

// One look-back wait on slot 0 of a cleared flag array: nothing publishes it,
// so the bounded wait gives up, latches the timeout error and returns.
__global__ void lookback_selftest_kernel(const u64 *flags, float2 *out) {
  if (threadIdx.x == 0) *out = lookback_const(flags, 1, cone());
}

// ------------------------------------------------------------- FBT
// Every product is bounded by dividing first, so absurd shapes cannot wrap
// around int64 and pass: rows x tiles must fit the 31-bit ticket counter.
int fbt_dims_ok(int64_t F, int64_t B, int64_t T) {
  if (F < 0 || B < 0 || T < 0) return RQF_ERR_SHAPE;
  if (B > 0x7fffffffLL || F > kMaxTickets || T > (1LL << 62)) return RQF_ERR_SHAPE;
  if (F == 0 || B == 0 || T == 0) return RQF_OK;
  if (F > kMaxTickets / B) return RQF_ERR_SHAPE;
  if (ceil_div(T, kFbtTile) > kMaxTickets / (F * B)) return RQF_ERR_SHAPE;
  return RQF_OK;
}

FbtArgs fbt_args(const float *c1, const float *tap0, const float *tap1, const float *z,
                 const float *gout, float *out, float *out2, float *carries, void *scratch,
                 int64_t F, int64_t B, int64_t T) {
  FbtArgs a;
  a.c1 = reinterpret_cast<const float2 *>(c1);
  a.tap0 = reinterpret_cast<const float2 *>(tap0);
  a.tap1 = reinterpret_cast<const float2 *>(tap1);
  a.z = reinterpret_cast<const float2 *>(z);
  a.gout = reinterpret_cast<const float2 *>(gout);
  a.skip = nullptr;
  a.out = reinterpret_cast<float2 *>(out);
  a.out2 = reinterpret_cast<float2 *>(out2);
  a.wsum = 0;
  a.carries = reinterpret_cast<float2 *>(carries);
  a.rows = F * B;
  a.T = T;
  a.batch = (int)B;
  a.ntiles = (int)ceil_div(T, kFbtTile);
  a.log2L = kFbtLog2Tile;
  const Scratch lay = scratch_layout(a.rows, a.ntiles);
  a.ticket = at<unsigned>(scratch, 0);
  a.flags = at<u64>(scratch, lay.flags_off);
  a.partials = at<float2>(scratch, lay.partials_off);
  return a;
}

// ------------------------------------------------------------- BTF
int btf_dims_ok(int64_t B, int64_t T, int64_t F) {
  if (B < 0 || T < 0 || F < 0) return RQF_ERR_SHAPE;
  if (B > 0 && F > 0 && btf_nsub(T) * B * ceil_div(F, 32) > kMaxTickets) return RQF_ERR_SHAPE;
  return RQF_OK;
}

// Arguments of one launch whose tiles are 2^log2S sub-tiles.
BtfArgs btf_args(const float *c1, const float *c2, const float *tap1, const void *x,
                 const float *gout, void *out, float *out2, float *carries, void *scratch,
                 int64_t B, int64_t T, int64_t F, int log2S) {
  BtfArgs a;
  a.c1 = reinterpret_cast<const float2 *>(c1);
  a.c2 = reinterpret_cast<const float2 *>(c2);
  a.tap1 = reinterpret_cast<const float2 *>(tap1);
  a.x = x;
  a.gout = reinterpret_cast<const float2 *>(gout);
  a.out = out;
  a.out2 = reinterpret_cast<float2 *>(out2);
  a.carries = reinterpret_cast<float2 *>(carries);
  a.B = B;
  a.T = T;
  a.F = F;
  a.nfb = (int)ceil_div(F, 32);
  a.ngroups = (int)(B * a.nfb);
  a.nsub = (int)btf_nsub(T);
  a.log2S = log2S;
  a.S = 1 << log2S;
  a.ntiles = (int)ceil_div(a.nsub, a.S);
  const BtfScratch lay = btf_scratch_layout(B, T, F);
  a.ticket = at<unsigned>(scratch, 0);
  a.flags = at<u64>(scratch, lay.base.flags_off);
  a.partials = at<float2>(scratch, lay.base.partials_off);
  a.pw = at<float2>(scratch, lay.pw_off);
  a.cw = nullptr;
  a.partials2 = nullptr;
  a.Fin = F;
  a.log2n = 0;
  return a;
}

// Clears the ticket and flags, fills the power table, and launches a (B,T,F)
// kernel with one CTA per tile.
template <typename Kern>
int btf_launch(Kern kernel, size_t smem, const BtfArgs &a, void *scratch, cudaStream_t stream) {
  const BtfScratch lay = btf_scratch_layout(a.B, a.T, a.F);
  int st = clear_lookback(scratch, lay.base, stream);
  if (st != RQF_OK) return st;
  btf_pow_table_kernel<<<(unsigned)ceil_div(a.F, 128), 128, 0, stream>>>(
      a.c1, const_cast<float2 *>(a.pw), a.F);
  if ((st = launch_status()) != RQF_OK) return st;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return RQF_ERR_LAUNCH;
  const int64_t tiles = (int64_t)a.ngroups * a.ntiles;
  kernel<<<(unsigned)tiles, kBtfThreads, smem, stream>>>(a);
  return launch_status();
}

template <int DRIVE, bool VEC, bool ABS = false, bool MOSC = false>
int btf_launch_fwd(const BtfArgs &a, void *scratch, cudaStream_t stream) {
  switch (a.S) {
    case 1:
      return btf_launch(btf_fwd_kernel<DRIVE, VEC, 1, ABS, MOSC>, btf_fwd_smem<DRIVE, 1>(), a,
                        scratch, stream);
    case 2:
      return btf_launch(btf_fwd_kernel<DRIVE, VEC, 2, ABS, MOSC>, btf_fwd_smem<DRIVE, 2>(), a,
                        scratch, stream);
    default:
      return btf_launch(btf_fwd_kernel<DRIVE, VEC, 4, ABS, MOSC>, btf_fwd_smem<DRIVE, 4>(), a,
                        scratch, stream);
  }
}

template <int DRIVE, bool VECX, bool VECG, bool MOSC = false>
int btf_launch_bwd(const BtfArgs &a, void *scratch, cudaStream_t stream) {
  if (a.S == 1)
    return btf_launch(btf_bwd_kernel<DRIVE, VECX, VECG, 1, MOSC>, btf_bwd_smem<DRIVE, 1>(), a,
                      scratch, stream);
  return btf_launch(btf_bwd_kernel<DRIVE, VECX, VECG, 2, MOSC>, btf_bwd_smem<DRIVE, 2>(), a,
                    scratch, stream);
}

// ---- multi-oscillator scans (tile-resident family only): Fin filters of
// num_osc oscillators each, lanes = oscillators.  Scratch: the BTF layout of
// the Fin * num_osc oscillator channels, then the C-weight partials.
inline int mosc_log2(int64_t n) {
  for (int l = 0; l <= 5; ++l)
    if ((int64_t)1 << l == n) return l;
  return -1;
}
struct MoscScratch {
  BtfScratch base;
  size_t p2_off, total;
};
inline MoscScratch mosc_scratch_layout(int64_t B, int64_t T, int64_t Fs) {
  MoscScratch m;
  m.base = btf_scratch_layout(B, T, Fs);
  m.p2_off = m.base.total;
  m.total = m.p2_off + round256((size_t)(B * Fs) * (size_t)btf_nsub(T) * 3 * sizeof(float2));
  return m;
}
BtfArgs mosc_args(const float *c1, const float *c2, const float *cw, const void *u,
                  const float *gout, void *out, float *carries, void *scratch, int64_t B,
                  int64_t T, int64_t Fin, int log2n, int max_log2_tile) {
  const int64_t Fs = Fin << log2n;
  BtfArgs a = btf_args(c1, c2, nullptr, u, gout, out, nullptr, carries, scratch, B, T, Fs,
                       btf_log2_tile(B, T, Fs, max_log2_tile));
  a.cw = reinterpret_cast<const float2 *>(cw);
  a.partials2 = at<float2>(scratch, mosc_scratch_layout(B, T, Fs).p2_off);
  a.Fin = Fin;
  a.log2n = log2n;
  return a;
}

// 16-byte staging copies: the row of a chain starts on a 16-byte boundary.
inline bool btf_vec(const void *p, int64_t F, size_t elem) {
  return p && aligned(p, 16) && (F * (int64_t)elem) % 16 == 0;
}

// ---- streaming path (rqf::btfs): few long chains.  Tiles of S x 128 steps
// re-read from L2 in their second pass, so a chain advances up to 1024 steps
// per look-back; the tile-resident kernels above hold a tile in shared memory
// and win when there are enough chains to keep the look-backs short.
namespace bs = rqf::btfs;
constexpr int kBtfsFwdWarps = 8, kBtfsFwdK = 16;
constexpr int kBtfsBwdWarps = 16, kBtfsBwdK = 8;
static_assert(kBtfsFwdWarps * kBtfsFwdK == bs::kBtfSub, "streaming forward sub-tile");
static_assert(kBtfsBwdWarps * kBtfsBwdK == bs::kBtfSub, "streaming backward sub-tile");
constexpr int64_t kBtfStreamChains = 48;  // chains below which the streaming path is used

// path: 0 automatic (by the number of chains), 1 streaming, 2 tile-resident.
// Passed per call; a backward must get the path its forward got (the saved
// entry states of the two families differ), which the automatic choice
// guarantees by itself since it depends only on the batch and filter counts.
inline bool btf_path_ok(int path) { return path >= 0 && path <= 2; }
inline bool btf_streaming(int64_t B, int64_t F, int path) {
  if (path != 0) return path == 1;
  return B * ceil_div(F, 32) < kBtfStreamChains;
}

// Sub-tiles (128 steps) per streaming tile: ngroups * S >= 80, S = 1..8.
inline int btfs_subtiles(int64_t B, int64_t F) {
  const int64_t groups = B * ceil_div(F, 32);
  int s = 1;
  while (s < bs::kBtfMaxS && groups * s < 80) s *= 2;
  return s;
}

bs::BtfArgs btfs_args(const float *c1, const float *c2, const float *tap1, const void *x,
                      const float *gout, void *out, float *out2, float *carries, void *scratch,
                      int64_t B, int64_t T, int64_t F) {
  bs::BtfArgs a;
  a.c1 = reinterpret_cast<const float2 *>(c1);
  a.c2 = reinterpret_cast<const float2 *>(c2);
  a.tap1 = reinterpret_cast<const float2 *>(tap1);
  a.x = x;
  a.gout = reinterpret_cast<const float2 *>(gout);
  a.out = out;
  a.out2 = reinterpret_cast<float2 *>(out2);
  a.carries = reinterpret_cast<float2 *>(carries);
  a.csub = (int)btf_nsub(T);  // row stride of the carry buffer: 64-step sub-tiles, so every
                              // 128-step one that starts before T has a slot
  a.B = B;
  a.T = T;
  a.F = F;
  a.nfb = (int)ceil_div(F, 32);
  a.ngroups = (int)(B * a.nfb);
  const int S = btfs_subtiles(B, F);
  a.ntiles = (int)ceil_div(T, (int64_t)bs::kBtfSub * S);
  a.log2L = bs::kBtfLog2Sub + (S == 1 ? 0 : S == 2 ? 1 : S == 4 ? 2 : 3);
  const Scratch lay = scratch_layout(B * F, a.ntiles);
  a.ticket = at<unsigned>(scratch, 0);
  a.flags = at<u64>(scratch, lay.flags_off);
  a.partials = at<float2>(scratch, lay.partials_off);
  return a;
}

// One streaming kernel: KIND 0 forward, 1 backward, 2 TBPTT(1) backward.
template <int KIND, int DRIVE, int S, bool ABS>
void btfs_kernel(const bs::BtfArgs &a, unsigned grid, cudaStream_t st) {
  if constexpr (KIND == 0)
    bs::btf_fwd_kernel<kBtfsFwdWarps, kBtfsFwdK, S, DRIVE, ABS>
        <<<grid, kBtfsFwdWarps * 32, 0, st>>>(a);
  else if constexpr (KIND == 1)
    bs::btf_bwd_kernel<kBtfsBwdWarps, kBtfsBwdK, S, DRIVE><<<grid, kBtfsBwdWarps * 32, 0, st>>>(a);
  else
    bs::btf_tbptt_bwd_kernel<kBtfsBwdWarps, kBtfsBwdK, S, false>
        <<<grid, kBtfsBwdWarps * 32, 0, st>>>(a);
}

// Launches a streaming kernel over all tiles after clearing the ticket and flags.
template <int KIND, int DRIVE, bool ABS = false>
int btfs_launch(const bs::BtfArgs &a, void *scratch, cudaStream_t st) {
  const int rc = clear_lookback(scratch, scratch_layout(a.B * a.F, a.ntiles), st);
  if (rc != RQF_OK) return rc;
  const unsigned grid = (unsigned)((int64_t)a.ngroups * a.ntiles);
  switch (btfs_subtiles(a.B, a.F)) {
    case 1: btfs_kernel<KIND, DRIVE, 1, ABS>(a, grid, st); break;
    case 2: btfs_kernel<KIND, DRIVE, 2, ABS>(a, grid, st); break;
    case 4: btfs_kernel<KIND, DRIVE, 4, ABS>(a, grid, st); break;
    default: btfs_kernel<KIND, DRIVE, 8, ABS>(a, grid, st); break;
  }
  return launch_status();
}

// Forward of one drive in one family; ABS writes |y| (float) and saves no carries.
template <int DRIVE, bool ABS>
int btf_forward_drive(const float *c1, const float *c2, const float *tap1, const void *x, void *y,
                      float *carries, void *scratch, int64_t B, int64_t T, int64_t F, int path,
                      cudaStream_t stream) {
  if (btf_streaming(B, F, path)) {
    const bs::BtfArgs sa = btfs_args(c1, c2, tap1, x, nullptr, y, nullptr, carries, scratch, B, T, F);
    return btfs_launch<0, DRIVE, ABS>(sa, scratch, stream);
  }
  const BtfArgs a = btf_args(c1, c2, tap1, x, nullptr, y, nullptr, carries, scratch, B, T, F,
                             btf_log2_tile(B, T, F, 2));
  const bool vec = btf_vec(x, F, DRIVE == kReal ? 4 : 8);
  return vec ? btf_launch_fwd<DRIVE, true, ABS>(a, scratch, stream)
             : btf_launch_fwd<DRIVE, false, ABS>(a, scratch, stream);
}

int btf_forward(int drive, const float *c1, const float *c2, const float *tap1, const void *x,
                void *y, float *carries, void *scratch, int64_t B, int64_t T, int64_t F,
                int path, cudaStream_t stream, bool abs_out = false) {
  if (!btf_path_ok(path)) return RQF_ERR_ARGUMENT;
  int st = btf_dims_ok(B, T, F);
  if (st != RQF_OK) return st;
  if (B == 0 || T == 0 || F == 0) return RQF_OK;
  if (!c1 || !c2 || !x || !y || (!carries && !abs_out) || !scratch ||
      (drive == kTwoTap && !tap1) || (abs_out && drive == kTwoTap))
    return RQF_ERR_ARGUMENT;
  if (!aligned(c1, 8) || !aligned(c2, 8) || !aligned(y, abs_out ? 4 : 8) ||
      (carries && !aligned(carries, 8)) || !aligned(scratch, 16) ||
      !aligned(x, drive == kReal ? 4 : 8) || (tap1 && !aligned(tap1, 8)))
    return RQF_ERR_ALIGN;
  if (abs_out)
    return drive == kReal
               ? btf_forward_drive<kReal, true>(c1, c2, tap1, x, y, nullptr, scratch, B, T, F, path,
                                                stream)
               : btf_forward_drive<kPlain, true>(c1, c2, tap1, x, y, nullptr, scratch, B, T, F,
                                                 path, stream);
  if (drive == kReal)
    return btf_forward_drive<kReal, false>(c1, c2, tap1, x, y, carries, scratch, B, T, F, path,
                                           stream);
  if (drive == kPlain)
    return btf_forward_drive<kPlain, false>(c1, c2, tap1, x, y, carries, scratch, B, T, F, path,
                                            stream);
  return btf_forward_drive<kTwoTap, false>(c1, c2, tap1, x, y, carries, scratch, B, T, F, path,
                                           stream);
}

template <int DRIVE>
int btf_backward_drive(const BtfArgs &a, bool vecx, bool vecg, void *scratch,
                       cudaStream_t stream) {
  if (vecx && vecg) return btf_launch_bwd<DRIVE, true, true>(a, scratch, stream);
  if (vecg) return btf_launch_bwd<DRIVE, false, true>(a, scratch, stream);
  return btf_launch_bwd<DRIVE, false, false>(a, scratch, stream);
}

int btf_backward(int drive, const float *c1, const float *c2, const float *tap1, const void *x,
                 const float *carries, const float *gy, void *gx, float *o0, float *o1,
                 float *o2, void *scratch, int64_t B, int64_t T, int64_t F, int path,
                 cudaStream_t stream) {
  if (!btf_path_ok(path)) return RQF_ERR_ARGUMENT;
  int st = btf_dims_ok(B, T, F);
  if (st != RQF_OK) return st;
  if (F == 0) return RQF_OK;
  if (B == 0 || T == 0) {
    if ((st = zero_complex(o0, F, stream)) != RQF_OK) return st;
    if ((st = zero_complex(o1, F, stream)) != RQF_OK) return st;
    return zero_complex(o2, F, stream);
  }
  if (!c1 || !c2 || !x || !carries || !gy || !gx || !scratch || (drive == kTwoTap && !tap1))
    return RQF_ERR_ARGUMENT;
  if (!aligned(c1, 8) || !aligned(c2, 8) || !aligned(gy, 8) || !aligned(carries, 8) ||
      !aligned(scratch, 16) || !aligned(x, drive == kReal ? 4 : 8) ||
      !aligned(gx, drive == kReal ? 4 : 8) || (tap1 && !aligned(tap1, 8)))
    return RQF_ERR_ALIGN;
  if (btf_streaming(B, F, path)) {
    const bs::BtfArgs sa = btfs_args(c1, c2, tap1, x, gy, gx, nullptr,
                                     const_cast<float *>(carries), scratch, B, T, F);
    st = drive == kReal    ? btfs_launch<1, kReal>(sa, scratch, stream)
         : drive == kPlain ? btfs_launch<1, kPlain>(sa, scratch, stream)
                           : btfs_launch<1, kTwoTap>(sa, scratch, stream);
    if (st != RQF_OK) return st;
    reduce_partials_kernel<<<(unsigned)F, 256, 0, stream>>>(
        sa.partials, reinterpret_cast<float2 *>(o0), reinterpret_cast<float2 *>(o1),
        reinterpret_cast<float2 *>(o2), B, 1, F, sa.ntiles);
    return launch_status();
  }
  const BtfArgs a = btf_args(c1, c2, tap1, x, gy, gx, nullptr, const_cast<float *>(carries),
                             scratch, B, T, F, btf_log2_tile(B, T, F, 1));
  const bool vecg = btf_vec(gy, F, 8);
  if (drive == kReal)
    st = btf_backward_drive<kReal>(a, btf_vec(x, F, 4), vecg, scratch, stream);
  else if (drive == kPlain)
    st = btf_backward_drive<kPlain>(a, btf_vec(x, F, 8), vecg, scratch, stream);
  else
    st = btf_backward_drive<kTwoTap>(a, btf_vec(x, F, 8), vecg, scratch, stream);
  if (st != RQF_OK) return st;
  reduce_partials_kernel<<<(unsigned)F, 256, 0, stream>>>(
      a.partials, reinterpret_cast<float2 *>(o0), reinterpret_cast<float2 *>(o1),
      reinterpret_cast<float2 *>(o2), B, 1, F, a.ntiles);
  return launch_status();
}

}  // namespace

extern "C" {

int rqf_abi_version(void) { return kAbiVersion; }

const char *rqf_status_string(int status) {
  switch (status) {
    case RQF_OK:
      return "ok";
    case RQF_ERR_SHAPE:
      return "invalid or unsupported shape";
    case RQF_ERR_ALIGN:
      return "pointer alignment requirement violated";
    case RQF_ERR_LOOKBACK_TIMEOUT:
      return "cross-tile look-back wait timed out";
    case RQF_ERR_LAUNCH:
      return "CUDA launch or memset failed";
    case RQF_ERR_ARGUMENT:
      return "null pointer or unsupported option";
    case RQF_ERR_CAPACITY:
      return "size exceeds the fixed internal maximum";
    case RQF_ERR_PIPELINE_TIMEOUT:
      return "tensor-core pipeline wait timed out";
    default:
      return "unknown status";
  }
}

int rqf_read_device_error(int *out_code, int clear, rqf_stream_t stream) {
  if (!out_code) return RQF_ERR_ARGUMENT;
  int h = 0;
  if (cudaMemcpyFromSymbolAsync(&h, g_rqf_error, sizeof(int), 0, cudaMemcpyDeviceToHost,
                                stream) != cudaSuccess)
    return RQF_ERR_LAUNCH;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return RQF_ERR_LAUNCH;
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbolAsync(g_rqf_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice,
                                stream) != cudaSuccess)
      return RQF_ERR_LAUNCH;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return RQF_ERR_LAUNCH;
  }
  *out_code = h;
  return RQF_OK;
}

int rqf_selftest_lookback_timeout(void *scratch, rqf_stream_t stream) {
  if (!scratch) return RQF_ERR_ARGUMENT;
  if (!aligned(scratch, 16)) return RQF_ERR_ALIGN;
  if (cudaMemsetAsync(scratch, 0, 256, stream) != cudaSuccess) return RQF_ERR_LAUNCH;
  u64 *flags = static_cast<u64 *>(scratch);
  float2 *out = reinterpret_cast<float2 *>(static_cast<char *>(scratch) + 128);
  lookback_selftest_kernel<<<1, 32, 0, stream>>>(flags, out);
  return launch_status();
}

// ---------------------------------------------------------------- sizes

int64_t rqf_btf_num_tiles(int64_t time) { return btf_nsub(time); }
int64_t rqf_btf_carry_count(int64_t batch, int64_t time, int64_t filters) {
  return batch * filters * btf_nsub(time);
}
size_t rqf_btf_scratch_bytes(int64_t batch, int64_t time, int64_t filters) {
  if (batch <= 0 || time <= 0 || filters <= 0) return 256;
  return btf_scratch_layout(batch, time, filters).total;
}
int64_t rqf_fbt_num_tiles(int64_t time) { return time <= 0 ? 0 : ceil_div(time, kFbtTile); }
int64_t rqf_fbt_carry_count(int64_t filters, int64_t batch, int64_t time) {
  if (fbt_dims_ok(filters, batch, time) != RQF_OK) return 0;
  // per-thread entry states of every tile, plus the marker element
  return fbt_marker(filters * batch, (int)rqf_fbt_num_tiles(time)) + 1;
}
size_t rqf_fbt_scratch_bytes(int64_t filters, int64_t batch, int64_t time) {
  if (fbt_dims_ok(filters, batch, time) != RQF_OK) return SIZE_MAX;  // no such launch
  if (batch <= 0 || time <= 0 || filters <= 0) return 256;
  return scratch_layout(filters * batch, rqf_fbt_num_tiles(time)).total;
}

// --------------------------------------------------------- BTF scans
int rqf_chunked_scan_forward(const float *c1, const float *c2, const void *u, int u_is_real,
                             float *y, float *carries, void *scratch, int64_t batch,
                             int64_t time, int64_t filters, int path, rqf_stream_t stream) {
  return btf_forward(u_is_real ? kReal : kPlain, c1, c2, nullptr, u, y, carries, scratch, batch,
                     time, filters, path, stream);
}

int rqf_chunked_scan_abs_forward(const float *c1, const float *c2, const void *u, int u_is_real,
                                 float *y_abs, void *scratch, int64_t batch, int64_t time,
                                 int64_t filters, int path, rqf_stream_t stream) {
  return btf_forward(u_is_real ? kReal : kPlain, c1, c2, nullptr, u, y_abs, nullptr, scratch,
                     batch, time, filters, path, stream, true);
}

int rqf_multi_osc_forward(const float *c1, const float *c2, const float *cw, const void *u,
                          int u_is_real, void *out, int out_abs, float *carries, void *scratch,
                          int64_t batch, int64_t time, int64_t filters, int64_t num_osc,
                          rqf_stream_t stream) {
  const int l = mosc_log2(num_osc);
  if (batch < 0 || time < 0 || filters < 0 || l < 0) return RQF_ERR_SHAPE;
  int st = btf_dims_ok(batch, time, filters << l);
  if (st != RQF_OK) return st;
  if (batch == 0 || time == 0 || filters == 0) return RQF_OK;
  if (!c1 || !c2 || !cw || !u || !out || (!carries && !out_abs) || !scratch)
    return RQF_ERR_ARGUMENT;
  if (!aligned(c1, 8) || !aligned(c2, 8) || !aligned(cw, 8) || !aligned(u, u_is_real ? 4 : 8) ||
      !aligned(out, out_abs ? 4 : 8) || (carries && !aligned(carries, 8)) ||
      !aligned(scratch, 16))
    return RQF_ERR_ALIGN;
  const BtfArgs a = mosc_args(c1, c2, cw, u, nullptr, out, out_abs ? nullptr : carries, scratch,
                              batch, time, filters, l, 2);
  if (u_is_real)
    return out_abs ? btf_launch_fwd<kReal, false, true, true>(a, scratch, stream)
                   : btf_launch_fwd<kReal, false, false, true>(a, scratch, stream);
  return out_abs ? btf_launch_fwd<kPlain, false, true, true>(a, scratch, stream)
                 : btf_launch_fwd<kPlain, false, false, true>(a, scratch, stream);
}

int rqf_multi_osc_backward(const float *c1, const float *c2, const float *cw, const void *u,
                           int u_is_real, const float *carries, const float *grad_out,
                           void *grad_u, float *grad_c1, float *grad_c2, float *grad_cw,
                           void *scratch, int64_t batch, int64_t time, int64_t filters,
                           int64_t num_osc, rqf_stream_t stream) {
  const int l = mosc_log2(num_osc);
  if (batch < 0 || time < 0 || filters < 0 || l < 0) return RQF_ERR_SHAPE;
  const int64_t Fs = filters << l;
  int st = btf_dims_ok(batch, time, Fs);
  if (st != RQF_OK) return st;
  if (filters == 0) return RQF_OK;
  if (batch == 0 || time == 0) {
    if ((st = zero_complex(grad_c1, Fs, stream)) != RQF_OK) return st;
    if ((st = zero_complex(grad_c2, Fs, stream)) != RQF_OK) return st;
    return zero_complex(grad_cw, Fs, stream);
  }
  if (!c1 || !c2 || !cw || !u || !carries || !grad_out || !grad_u || !scratch)
    return RQF_ERR_ARGUMENT;
  if (!aligned(c1, 8) || !aligned(c2, 8) || !aligned(cw, 8) || !aligned(u, u_is_real ? 4 : 8) ||
      !aligned(grad_out, 8) || !aligned(grad_u, u_is_real ? 4 : 8) || !aligned(carries, 8) ||
      !aligned(scratch, 16))
    return RQF_ERR_ALIGN;
  const BtfArgs a = mosc_args(c1, c2, cw, u, grad_out, grad_u, const_cast<float *>(carries),
                              scratch, batch, time, filters, l, 1);
  st = u_is_real ? btf_launch_bwd<kReal, false, false, true>(a, scratch, stream)
                 : btf_launch_bwd<kPlain, false, false, true>(a, scratch, stream);
  if (st != RQF_OK) return st;
  reduce_partials_kernel<<<(unsigned)Fs, 256, 0, stream>>>(
      a.partials, reinterpret_cast<float2 *>(grad_c1), reinterpret_cast<float2 *>(grad_c2),
      nullptr, batch, 1, Fs, a.ntiles);
  if ((st = launch_status()) != RQF_OK) return st;
  reduce_partials_kernel<<<(unsigned)Fs, 256, 0, stream>>>(
      a.partials2, reinterpret_cast<float2 *>(grad_cw), nullptr, nullptr, batch, 1, Fs,
      a.ntiles);
  return launch_status();
}

int64_t rqf_multi_osc_carry_count(int64_t batch, int64_t time, int64_t filters,
                                  int64_t num_osc) {
  const int l = mosc_log2(num_osc);
  if (l < 0 || batch < 0 || time < 0 || filters < 0) return 0;
  return batch * (filters << l) * btf_nsub(time);
}

size_t rqf_multi_osc_scratch_bytes(int64_t batch, int64_t time, int64_t filters,
                                   int64_t num_osc) {
  const int l = mosc_log2(num_osc);
  if (l < 0 || batch <= 0 || time <= 0 || filters <= 0) return 256;
  return mosc_scratch_layout(batch, time, filters << l).total;
}

int rqf_chunked_scan_backward(const float *c1, const float *c2, const void *u, int u_is_real,
                              const float *carries, const float *grad_y, void *grad_u,
                              float *grad_c1, float *grad_c2, void *scratch, int64_t batch,
                              int64_t time, int64_t filters, int path, rqf_stream_t stream) {
  return btf_backward(u_is_real ? kReal : kPlain, c1, c2, nullptr, u, carries, grad_y, grad_u,
                      grad_c1, grad_c2, nullptr, scratch, batch, time, filters, path, stream);
}

int rqf_chunked_prospective_forward(const float *c1, const float *tap0, const float *tap1,
                                    const float *x, float *y, float *carries, void *scratch,
                                    int64_t batch, int64_t time, int64_t filters, int path,
                                    rqf_stream_t stream) {
  return btf_forward(kTwoTap, c1, tap0, tap1, x, y, carries, scratch, batch, time, filters,
                     path, stream);
}

int rqf_chunked_prospective_backward(const float *c1, const float *tap0, const float *tap1,
                                     const float *x, const float *carries, const float *grad_y,
                                     float *grad_x, float *grad_c1, float *grad_tap0,
                                     float *grad_tap1, void *scratch, int64_t batch,
                                     int64_t time, int64_t filters, int path,
                                     rqf_stream_t stream) {
  return btf_backward(kTwoTap, c1, tap0, tap1, x, carries, grad_y, grad_x, grad_c1, grad_tap0,
                      grad_tap1, scratch, batch, time, filters, path, stream);
}

// --------------------------------------------------------- FBT scans
int rqf_fbt_prospective_forward(const float *c1, const float *tap0, const float *tap1,
                                const float *z, float *out, float *carries, void *scratch,
                                int64_t filters, int64_t batch, int64_t time, int fuse_act,
                                rqf_stream_t stream) {
  return rqf_fbt_block_forward(c1, tap0, tap1, z, nullptr, out, carries, scratch, filters, batch,
                               time, fuse_act, stream);
}

int rqf_fbt_block_forward(const float *c1, const float *tap0, const float *tap1, const float *z,
                          const float *skip, float *out, float *carries, void *scratch,
                          int64_t filters, int64_t batch, int64_t time, int fuse_act,
                          rqf_stream_t stream) {
  int st = fbt_dims_ok(filters, batch, time);
  if (st != RQF_OK) return st;
  if (filters == 0 || batch == 0 || time == 0) return RQF_OK;
  if (!c1 || !tap0 || !tap1 || !z || !out || !carries || !scratch) return RQF_ERR_ARGUMENT;
  if (!aligned(c1, 8) || !aligned(tap0, 8) || !aligned(tap1, 8) || !aligned(z, 8) ||
      !aligned(out, 8) || !aligned(carries, 8) || !aligned(scratch, 16) ||
      (skip && !aligned(skip, 8)))
    return RQF_ERR_ALIGN;
  FbtArgs a = fbt_args(c1, tap0, tap1, z, nullptr, out, nullptr, carries, scratch, filters,
                       batch, time);
  a.skip = reinterpret_cast<const float2 *>(skip);
  const bool vec =
      (time % 2 == 0) && aligned(z, 16) && aligned(out, 16) && (!skip || aligned(skip, 16));
  if (vec) {
    bool done;
    if (skip) {
      constexpr size_t smem = fbt_rows_smem_bytes<kFbtThreads, kFbtK, 2, kRowsBwdStages>();
      done = fuse_act ? launch_rows(fbt_fwd_rows_kernel<kFbtThreads, kFbtK, kRowsBwdStages, true,
                                                        true>, smem, a, stream)
                      : launch_rows(fbt_fwd_rows_kernel<kFbtThreads, kFbtK, kRowsBwdStages,
                                                        false, true>, smem, a, stream);
    } else {
      constexpr size_t smem = fbt_rows_smem_bytes<kFbtThreads, kFbtK, 1, kRowsFwdStages>();
      done = fuse_act ? launch_rows(fbt_fwd_rows_kernel<kFbtThreads, kFbtK, kRowsFwdStages, true>,
                                    smem, a, stream)
                      : launch_rows(fbt_fwd_rows_kernel<kFbtThreads, kFbtK, kRowsFwdStages, false>,
                                    smem, a, stream);
    }
    if (done) return launch_status();
  }
  const Scratch lay = scratch_layout(a.rows, a.ntiles);
  if ((st = clear_lookback(scratch, lay, stream)) != RQF_OK) return st;
  const unsigned grid = (unsigned)(a.rows * a.ntiles);
  if (vec) {
    if (fuse_act)
      fbt_fwd_kernel<kFbtThreads, kFbtK, true, true><<<grid, kFbtThreads, 0, stream>>>(a);
    else
      fbt_fwd_kernel<kFbtThreads, kFbtK, true, false><<<grid, kFbtThreads, 0, stream>>>(a);
  } else {
    if (fuse_act)
      fbt_fwd_kernel<kFbtThreads, kFbtK, false, true><<<grid, kFbtThreads, 0, stream>>>(a);
    else
      fbt_fwd_kernel<kFbtThreads, kFbtK, false, false><<<grid, kFbtThreads, 0, stream>>>(a);
  }
  return launch_status();
}

// ------------------------------------------------ rank-1 first block
}  // extern "C"

namespace {

constexpr int kRank1FwdStages = kRowsFwdStages, kRank1BwdStages = kRowsBwdStages;
constexpr size_t kRank1FwdSmem = fbt_rows_smem_bytes<kFbtThreads, kFbtK, 1, kRank1FwdStages>();
constexpr size_t kRank1BwdSmem = fbt_rows_smem_bytes<kFbtThreads, kFbtK, 2, kRank1BwdStages>();

// Both row kernels of the rank-1 block take the shape: enough rows for every
// resident CTA, T a multiple of 4 (16-byte x pieces), 32-bit cursors.
bool rank1_shape_ok(int64_t F, int64_t B, int64_t T) {
  if (fbt_dims_ok(F, B, T) != RQF_OK || F <= 0 || B <= 0 || T <= 0 || T % 4 != 0) return false;
  if (T > 0x7fffffffLL || F * B > 0x7fffffffLL) return false;
  const int64_t gf = resident_ctas(fbt_rank1_fwd_kernel<kFbtThreads, kFbtK, kRank1FwdStages, true>,
                                   kFbtThreads, kRank1FwdSmem);
  const int64_t gb = resident_ctas(
      fbt_rank1_bwd_kernel<kFbtThreads, kFbtK, kRank1BwdStages, true, true>, kFbtThreads,
      kRank1BwdSmem);
  return gf > 0 && gb > 0 && F * B >= gf && F * B >= gb;
}

}  // namespace

extern "C" {

int rqf_fbt_rank1_supported(int64_t filters, int64_t batch, int64_t time) {
  return rank1_shape_ok(filters, batch, time) ? 1 : 0;
}

size_t rqf_fbt_rank1_scratch_bytes(int64_t filters, int64_t batch, int64_t time) {
  if (fbt_dims_ok(filters, batch, time) != RQF_OK) return SIZE_MAX;
  return round256((size_t)filters * batch * 3 * sizeof(float2)) +
         round256((size_t)filters * batch * 6 * sizeof(float2));
}

int rqf_fbt_rank1_forward(const float *u, const float *beta, const float *w, const float *bb,
                          const float *x, const float *c1, const float *tap0, const float *tap1,
                          float *out, float *carries, int64_t filters, int64_t batch,
                          int64_t time, int fuse_act, rqf_stream_t stream) {
  int st = fbt_dims_ok(filters, batch, time);
  if (st != RQF_OK) return st;
  if (filters == 0 || batch == 0 || time == 0) return RQF_OK;
  if (!rank1_shape_ok(filters, batch, time)) return RQF_ERR_SHAPE;
  if (!u || !x || !c1 || !tap0 || !tap1 || !out || !carries) return RQF_ERR_ARGUMENT;
  if (!aligned(u, 8) || (beta && !aligned(beta, 8)) || !aligned(x, 16) || !aligned(c1, 8) ||
      !aligned(tap0, 8) || !aligned(tap1, 8) || !aligned(out, 16) || !aligned(carries, 8))
    return RQF_ERR_ALIGN;
  FbtArgs a = fbt_args(c1, tap0, tap1, nullptr, nullptr, out, nullptr, carries, nullptr, filters,
                       batch, time);
  Rank1Args r{reinterpret_cast<const float2 *>(u), reinterpret_cast<const float2 *>(beta), w, bb, x,
              nullptr};
  auto kern = fuse_act ? fbt_rank1_fwd_kernel<kFbtThreads, kFbtK, kRank1FwdStages, true>
                       : fbt_rank1_fwd_kernel<kFbtThreads, kFbtK, kRank1FwdStages, false>;
  const int64_t g = resident_ctas(kern, kFbtThreads, kRank1FwdSmem);
  kern<<<(unsigned)g, kFbtThreads, kRank1FwdSmem, reinterpret_cast<cudaStream_t>(stream)>>>(a, r);
  return launch_status();
}

extern "C++" {
namespace {
// Both rank-1 backwards: TRUNC the TBPTT(1) surrogate, which also returns gwx.
template <bool TRUNC>
int rank1_backward_impl(const float *u, const float *beta, const float *x, const float *c1,
                        const float *tap0, const float *tap1, const float *carries,
                        const float *grad_out, float *gzx, float *gwx, float *gsx, float *grad_c1,
                        float *grad_tap0, float *grad_tap1, void *scratch, int64_t filters,
                        int64_t batch, int64_t time, int fuse_act, int with_sum,
                        cudaStream_t sm) {
  int st = fbt_dims_ok(filters, batch, time);
  if (st != RQF_OK) return st;
  if (filters == 0) return RQF_OK;
  if (batch == 0 || time == 0) {
    for (float *p : {grad_c1, grad_tap0, grad_tap1})
      if ((st = zero_complex(p, filters, sm)) != RQF_OK) return st;
    if ((st = zero_complex(gzx, 2 * filters, sm)) != RQF_OK) return st;
    if ((st = zero_complex(gwx, 2 * filters, sm)) != RQF_OK) return st;
    return zero_complex(gsx, 2 * filters, sm);
  }
  if (!rank1_shape_ok(filters, batch, time)) return RQF_ERR_SHAPE;
  if (!u || !x || !c1 || !tap0 || !tap1 || !carries || !grad_out || !gzx || !grad_c1 ||
      !grad_tap0 || !grad_tap1 || !scratch || (TRUNC && !gwx))
    return RQF_ERR_ARGUMENT;
  if (!aligned(u, 8) || (beta && !aligned(beta, 8)) || !aligned(x, 16) || !aligned(c1, 8) ||
      !aligned(tap0, 8) || !aligned(tap1, 8) || !aligned(carries, 8) || !aligned(grad_out, 16) ||
      !aligned(gzx, 8) || (gsx && !aligned(gsx, 8)) || (gwx && !aligned(gwx, 8)) ||
      !aligned(scratch, 16))
    return RQF_ERR_ALIGN;
  FbtArgs a = fbt_args(c1, tap0, tap1, nullptr, grad_out, nullptr, nullptr,
                       const_cast<float *>(carries), nullptr, filters, batch, time);
  const int64_t rows = filters * batch;
  a.partials = static_cast<float2 *>(scratch);
  float2 *rowsums = at<float2>(scratch, round256((size_t)rows * 3 * sizeof(float2)));
  Rank1Args r{reinterpret_cast<const float2 *>(u), reinterpret_cast<const float2 *>(beta),
              nullptr, nullptr, x, rowsums};
  const bool wsum = with_sum != 0;
  constexpr int NT = kFbtThreads, K = kFbtK, S = kRank1BwdStages;
  auto kern = fuse_act ? (wsum ? fbt_rank1_bwd_kernel<NT, K, S, true, true, TRUNC>
                               : fbt_rank1_bwd_kernel<NT, K, S, true, false, TRUNC>)
                       : (wsum ? fbt_rank1_bwd_kernel<NT, K, S, false, true, TRUNC>
                               : fbt_rank1_bwd_kernel<NT, K, S, false, false, TRUNC>);
  const int64_t g = resident_ctas(kern, kFbtThreads, kRank1BwdSmem);
  kern<<<(unsigned)g, kFbtThreads, kRank1BwdSmem, sm>>>(a, r);
  if ((st = launch_status()) != RQF_OK) return st;
  reduce_partials_kernel<<<(unsigned)filters, 256, 0, sm>>>(
      a.partials, reinterpret_cast<float2 *>(grad_c1), reinterpret_cast<float2 *>(grad_tap0),
      reinterpret_cast<float2 *>(grad_tap1), batch, batch, 1, 1);
  if ((st = launch_status()) != RQF_OK) return st;
  // (F, 2) sums {gz x, gz} into gzx, {g x, g} into gsx and, TRUNC, {gsum x, gsum} into gwx
  const int R = TRUNC ? 6 : 4;
  reduce_rows4_kernel<<<(unsigned)ceil_div(filters * R, 256), 256, 0, sm>>>(
      rowsums, reinterpret_cast<float2 *>(gzx), reinterpret_cast<float2 *>(gsx),
      reinterpret_cast<float2 *>(gwx), filters, (int)batch, R);
  return launch_status();
}
}  // namespace
}  // extern "C++"

int rqf_fbt_rank1_backward(const float *u, const float *beta, const float *x, const float *c1,
                           const float *tap0, const float *tap1, const float *carries,
                           const float *grad_out, float *gzx, float *gsx, float *grad_c1,
                           float *grad_tap0, float *grad_tap1, void *scratch, int64_t filters,
                           int64_t batch, int64_t time, int fuse_act, int with_sum,
                           rqf_stream_t stream) {
  return rank1_backward_impl<false>(u, beta, x, c1, tap0, tap1, carries, grad_out, gzx, nullptr,
                                    gsx, grad_c1, grad_tap0, grad_tap1, scratch, filters, batch,
                                    time, fuse_act, with_sum,
                                    reinterpret_cast<cudaStream_t>(stream));
}

int rqf_fbt_rank1_tbptt_backward(const float *u, const float *beta, const float *x,
                                 const float *c1, const float *tap0, const float *tap1,
                                 const float *carries, const float *grad_out, float *gzx,
                                 float *gwx, float *gsx, float *grad_c1, float *grad_tap0,
                                 float *grad_tap1, void *scratch, int64_t filters, int64_t batch,
                                 int64_t time, int fuse_act, int with_sum, rqf_stream_t stream) {
  return rank1_backward_impl<true>(u, beta, x, c1, tap0, tap1, carries, grad_out, gzx, gwx, gsx,
                                   grad_c1, grad_tap0, grad_tap1, scratch, filters, batch, time,
                                   fuse_act, with_sum, reinterpret_cast<cudaStream_t>(stream));
}

int rqf_fbt_prospective_backward(const float *c1, const float *tap0, const float *tap1,
                                 const float *z, const float *carries, const float *grad_out,
                                 float *grad_z, float *grad_c1, float *grad_tap0,
                                 float *grad_tap1, void *scratch, int64_t filters, int64_t batch,
                                 int64_t time, int fuse_act, rqf_stream_t stream) {
  int st = fbt_dims_ok(filters, batch, time);
  if (st != RQF_OK) return st;
  if (filters == 0) return RQF_OK;
  if (batch == 0 || time == 0) {
    if ((st = zero_complex(grad_c1, filters, stream)) != RQF_OK) return st;
    if ((st = zero_complex(grad_tap0, filters, stream)) != RQF_OK) return st;
    return zero_complex(grad_tap1, filters, stream);
  }
  if (!c1 || !tap0 || !tap1 || !z || !carries || !grad_out || !grad_z || !scratch)
    return RQF_ERR_ARGUMENT;
  if (!aligned(c1, 8) || !aligned(tap0, 8) || !aligned(tap1, 8) || !aligned(z, 8) ||
      !aligned(grad_out, 8) || !aligned(grad_z, 8) || !aligned(carries, 8) ||
      !aligned(scratch, 16))
    return RQF_ERR_ALIGN;
  FbtArgs a = fbt_args(c1, tap0, tap1, z, grad_out, grad_z, nullptr, const_cast<float *>(carries),
                       scratch, filters, batch, time);
  const bool vec =
      (time % 2 == 0) && aligned(z, 16) && aligned(grad_out, 16) && aligned(grad_z, 16);
  if (vec) {
    constexpr size_t smem = fbt_rows_smem_bytes<kFbtThreads, kFbtK, 2, kRowsBwdStages>();
    const bool done =
        fuse_act ? launch_rows(fbt_bwd_rows_kernel<kFbtThreads, kFbtK, kRowsBwdStages, true>, smem,
                               a, stream)
                 : launch_rows(fbt_bwd_rows_kernel<kFbtThreads, kFbtK, kRowsBwdStages, false>,
                               smem, a, stream);
    if (done) {
      if ((st = launch_status()) != RQF_OK) return st;
      reduce_partials_kernel<<<(unsigned)filters, 256, 0, stream>>>(
          a.partials, reinterpret_cast<float2 *>(grad_c1), reinterpret_cast<float2 *>(grad_tap0),
          reinterpret_cast<float2 *>(grad_tap1), batch, batch, 1, 1);
      return launch_status();
    }
  }
  const Scratch lay = scratch_layout(a.rows, a.ntiles);
  if ((st = clear_lookback(scratch, lay, stream)) != RQF_OK) return st;
  const unsigned grid = (unsigned)(a.rows * a.ntiles);
  if (vec) {
    if (fuse_act)
      fbt_bwd_kernel<kFbtThreads, kFbtK, true, true><<<grid, kFbtThreads, 0, stream>>>(a);
    else
      fbt_bwd_kernel<kFbtThreads, kFbtK, true, false><<<grid, kFbtThreads, 0, stream>>>(a);
  } else {
    if (fuse_act)
      fbt_bwd_kernel<kFbtThreads, kFbtK, false, true><<<grid, kFbtThreads, 0, stream>>>(a);
    else
      fbt_bwd_kernel<kFbtThreads, kFbtK, false, false><<<grid, kFbtThreads, 0, stream>>>(a);
  }
  if ((st = launch_status()) != RQF_OK) return st;
  reduce_partials_kernel<<<(unsigned)filters, 256, 0, stream>>>(
      a.partials, reinterpret_cast<float2 *>(grad_c1), reinterpret_cast<float2 *>(grad_tap0),
      reinterpret_cast<float2 *>(grad_tap1), batch, batch, 1, a.ntiles);
  return launch_status();
}

// ------------------------------------------------------------ TBPTT(1)
// wsum (layout 1 only): grad_zw receives grad_z + grad_zw.
static int tbptt1_backward_impl(int layout, const float *c1, const float *tap0,
                                const float *tap1, const float *z, const float *carries,
                                const float *grad_out, float *grad_z, float *grad_zw,
                                float *grad_c1, float *grad_tap0, float *grad_tap1,
                                void *scratch, int64_t d0, int64_t d1, int64_t d2, int fuse_act,
                                int path, rqf_stream_t stream, int wsum) {
  if (layout != 0 && layout != 1) return RQF_ERR_ARGUMENT;
  if (wsum && layout != 1) return RQF_ERR_ARGUMENT;
  if (!btf_path_ok(path)) return RQF_ERR_ARGUMENT;
  const int64_t F = layout == 0 ? d2 : d0;
  const int64_t B = layout == 0 ? d0 : d1;
  const int64_t T = layout == 0 ? d1 : d2;
  int st = layout == 0 ? btf_dims_ok(B, T, F) : fbt_dims_ok(F, B, T);
  if (st != RQF_OK) return st;
  if (F == 0) return RQF_OK;
  if (B == 0 || T == 0) {
    if ((st = zero_complex(grad_c1, F, stream)) != RQF_OK) return st;
    if ((st = zero_complex(grad_tap0, F, stream)) != RQF_OK) return st;
    return zero_complex(grad_tap1, F, stream);
  }
  if (!c1 || !tap0 || !tap1 || !z || !carries || !grad_out || !grad_z || !grad_zw || !scratch)
    return RQF_ERR_ARGUMENT;
  if (!aligned(c1, 8) || !aligned(tap0, 8) || !aligned(tap1, 8) || !aligned(z, 8) ||
      !aligned(grad_out, 8) || !aligned(grad_z, 8) || !aligned(grad_zw, 8) ||
      !aligned(carries, 8) || !aligned(scratch, 16))
    return RQF_ERR_ALIGN;
  if (layout == 0) {
    // the (B,T,F) forward has no fused activation, so neither has its TBPTT(1) backward
    if (fuse_act) return RQF_ERR_ARGUMENT;
    if (btf_streaming(B, F, path)) {
      const bs::BtfArgs sa = btfs_args(c1, tap0, tap1, z, grad_out, grad_z, grad_zw,
                                       const_cast<float *>(carries), scratch, B, T, F);
      if ((st = btfs_launch<2, kTwoTap>(sa, scratch, stream)) != RQF_OK) return st;
      reduce_partials_kernel<<<(unsigned)F, 256, 0, stream>>>(
          sa.partials, reinterpret_cast<float2 *>(grad_c1), reinterpret_cast<float2 *>(grad_tap0),
          reinterpret_cast<float2 *>(grad_tap1), B, 1, F, sa.ntiles);
      return launch_status();
    }
    static_assert(kBtfTbpttS == 4, "TBPTT(1) tiles of 4 sub-tiles");
    const BtfArgs a = btf_args(c1, tap0, tap1, z, grad_out, grad_z, grad_zw,
                               const_cast<float *>(carries), scratch, B, T, F, 2);
    const bool vec = btf_vec(z, F, 8) && btf_vec(grad_out, F, 8);
    st = vec ? btf_launch(btf_tbptt_bwd_kernel<true>, btf_tbptt_smem(), a, scratch, stream)
             : btf_launch(btf_tbptt_bwd_kernel<false>, btf_tbptt_smem(), a, scratch, stream);
    if (st != RQF_OK) return st;
    reduce_partials_kernel<<<(unsigned)F, 256, 0, stream>>>(
        a.partials, reinterpret_cast<float2 *>(grad_c1), reinterpret_cast<float2 *>(grad_tap0),
        reinterpret_cast<float2 *>(grad_tap1), B, 1, F, a.ntiles);
    return launch_status();
  }
  FbtArgs a = fbt_args(c1, tap0, tap1, z, grad_out, grad_z, grad_zw, const_cast<float *>(carries),
                       scratch, F, B, T);
  a.wsum = wsum ? 1 : 0;
  const bool vec = (T % 2 == 0) && aligned(z, 16) && aligned(grad_out, 16) &&
                   aligned(grad_z, 16) && aligned(grad_zw, 16);
  if (vec) {
    constexpr size_t smem = fbt_rows_smem_bytes<kFbtThreads, kFbtK, 2, kRowsBwdStages>();
    const bool done =
        fuse_act ? launch_rows(fbt_tbptt_rows_kernel<kFbtThreads, kFbtK, kRowsBwdStages, true>,
                               smem, a, stream)
                 : launch_rows(fbt_tbptt_rows_kernel<kFbtThreads, kFbtK, kRowsBwdStages, false>,
                               smem, a, stream);
    if (done) {
      if ((st = launch_status()) != RQF_OK) return st;
      reduce_partials_kernel<<<(unsigned)F, 256, 0, stream>>>(
          a.partials, reinterpret_cast<float2 *>(grad_c1), reinterpret_cast<float2 *>(grad_tap0),
          reinterpret_cast<float2 *>(grad_tap1), B, B, 1, 1);
      return launch_status();
    }
  }
  const unsigned grid = (unsigned)(a.rows * a.ntiles);
  if (vec) {
    if (fuse_act)
      fbt_tbptt_bwd_kernel<kFbtThreads, kFbtK, true, true><<<grid, kFbtThreads, 0, stream>>>(a);
    else
      fbt_tbptt_bwd_kernel<kFbtThreads, kFbtK, true, false><<<grid, kFbtThreads, 0, stream>>>(a);
  } else {
    if (fuse_act)
      fbt_tbptt_bwd_kernel<kFbtThreads, kFbtK, false, true><<<grid, kFbtThreads, 0, stream>>>(a);
    else
      fbt_tbptt_bwd_kernel<kFbtThreads, kFbtK, false, false>
          <<<grid, kFbtThreads, 0, stream>>>(a);
  }
  if ((st = launch_status()) != RQF_OK) return st;
  reduce_partials_kernel<<<(unsigned)F, 256, 0, stream>>>(
      a.partials, reinterpret_cast<float2 *>(grad_c1), reinterpret_cast<float2 *>(grad_tap0),
      reinterpret_cast<float2 *>(grad_tap1), B, B, 1, a.ntiles);
  return launch_status();
}


int rqf_tbptt1_two_tap_backward(int layout, const float *c1, const float *tap0,
                                const float *tap1, const float *z, const float *carries,
                                const float *grad_out, float *grad_z, float *grad_zw,
                                float *grad_c1, float *grad_tap0, float *grad_tap1,
                                void *scratch, int64_t d0, int64_t d1, int64_t d2, int fuse_act,
                                int path, rqf_stream_t stream) {
  return tbptt1_backward_impl(layout, c1, tap0, tap1, z, carries, grad_out, grad_z, grad_zw,
                              grad_c1, grad_tap0, grad_tap1, scratch, d0, d1, d2, fuse_act, path,
                              stream, 0);
}

int rqf_fbt_tbptt1_backward_wsum(const float *c1, const float *tap0, const float *tap1,
                                 const float *z, const float *carries, const float *grad_out,
                                 float *grad_z, float *grad_zsum, float *grad_c1,
                                 float *grad_tap0, float *grad_tap1, void *scratch,
                                 int64_t filters, int64_t batch, int64_t time, int fuse_act,
                                 rqf_stream_t stream) {
  return tbptt1_backward_impl(1, c1, tap0, tap1, z, carries, grad_out, grad_z, grad_zsum,
                              grad_c1, grad_tap0, grad_tap1, scratch, filters, batch, time,
                              fuse_act, 0, stream, 1);
}
}  // extern "C"

// ------------------------------------------------------------ selective
namespace {

SelArgs sel_args(const float *z, const rqf_selective_inputs *in, const rqf_selective_options *o,
                 int64_t F, int64_t B, int64_t T) {
  SelArgs a = {};
  a.z = reinterpret_cast<const float2 *>(z);
  a.G = o->has_gamma ? in->gamma_logits : nullptr;
  a.D = o->has_warp ? in->warp_logits : nullptr;
  a.W = o->has_write ? in->write_logits : nullptr;
  a.bias = in->bias;
  a.theta = in->theta;
  a.groups = reinterpret_cast<const long long *>(in->groups);
  a.lo = in->minimum;
  a.span = in->span;
  a.step = in->step;
  a.horizon = in->horizon;
  a.th_lo = in->theta_minimum;
  a.th_hi = in->theta_maximum;
  a.rows = (int)(F * B);
  a.T = (int)T;
  a.batch = (int)B;
  a.ntiles = (int)ceil_div(T, kSelTile);
  a.num_groups = (int)in->num_groups;
  a.o.has_gamma = o->has_gamma;
  a.o.has_warp = o->has_warp;
  a.o.has_write = o->has_write;
  a.o.log_shift = o->log_shift;
  a.o.gamma_scale = o->gamma_scale;
  a.o.warp_scale = o->warp_scale;
  a.o.prospective = o->prospective;
  a.o.gamma_horizon = o->gamma_horizon;
  a.o.write_sigmoid = o->write_sigmoid;
  a.o.write_max = o->write_max;
  a.o.write_bias = o->write_bias;
  a.o.bound_warp = o->bound_warp;
  return a;
}

int sel_check(const float *z, const rqf_selective_inputs *in, const rqf_selective_options *o,
              int64_t F, int64_t B, int64_t T) {
  if (F < 0 || B < 0 || T < 0) return RQF_ERR_SHAPE;
  if (F * B > 0x7fffffffLL || T > 0x7fffffffLL) return RQF_ERR_SHAPE;
  if (!in || !o) return RQF_ERR_ARGUMENT;
  if (F * B * T == 0) return RQF_OK;
  if (!z || !in->bias || !in->theta || !in->minimum || !in->span || !in->step || !in->horizon ||
      !in->theta_minimum || !in->theta_maximum)
    return RQF_ERR_ARGUMENT;
  if ((o->has_gamma && !in->gamma_logits) || (o->has_write && !in->write_logits) ||
      (o->has_warp && (!in->warp_logits || !in->groups || in->num_groups < 1 ||
                       in->num_groups > 32)))
    return RQF_ERR_ARGUMENT;
  if (!aligned(z, 8)) return RQF_ERR_ALIGN;
  return RQF_OK;
}

// 16-byte per-thread accesses need every per-sample row to start on a
// 16-byte boundary: T a multiple of 4 and 16-byte aligned base pointers.
int sel_vec(const SelArgs &a, int64_t T) {
  if (T % 4 != 0) return 0;
  const void *ptrs[] = {a.z, a.G, a.D, a.W, a.raw, a.act, a.gy, a.gx, a.dz, a.dzw, a.dG, a.dD, a.dW};
  for (const void *p : ptrs)
    if (p != nullptr && !aligned(p, 16)) return 0;
  return 1;
}

template <typename Kern>
unsigned sel_grid(Kern kernel, int64_t rows) {
  const int64_t g = resident_ctas(kernel, kSelThreads, 0);
  const int64_t n = g > 0 ? (g < rows ? g : rows) : (rows < 1024 ? rows : 1024);
  return (unsigned)(n > 0 ? n : 1);
}

}  // namespace

extern "C" {

int64_t rqf_selective_num_tiles(int64_t time) { return time <= 0 ? 0 : ceil_div(time, kSelTile); }
int64_t rqf_selective_carry_count(int64_t filters, int64_t batch, int64_t time) {
  return filters * batch * rqf_selective_num_tiles(time);
}
size_t rqf_selective_scratch_bytes(int64_t filters, int64_t batch, int64_t time, int has_warp) {
  if (filters <= 0 || batch <= 0 || time <= 0) return 256;
  const size_t dd = has_warp ? round256((size_t)filters * batch * time * sizeof(float)) : 0;
  const size_t order = has_warp ? round256((size_t)(filters + 33) * sizeof(int)) : 0;
  return dd + round256((size_t)filters * batch * 2 * sizeof(float)) + order;
}

}  // extern "C"

namespace {

template <bool BF>
int sel_forward_impl(const float *z, const rqf_selective_inputs *inputs,
                     const rqf_selective_options *options, void *raw, void *act, float *carries,
                     int64_t filters, int64_t batch, int64_t time, rqf_stream_t stream) {
  int st = sel_check(z, inputs, options, filters, batch, time);
  if (st != RQF_OK || filters * batch * time == 0) return st;
  if ((!raw && !act) || !carries) return RQF_ERR_ARGUMENT;
  const size_t out_align = BF ? 4 : 8;
  if ((raw && !aligned(raw, out_align)) || (act && !aligned(act, out_align)) ||
      !aligned(carries, 8))
    return RQF_ERR_ALIGN;
  SelArgs a = sel_args(z, inputs, options, filters, batch, time);
  a.raw = raw;
  a.act = act;
  a.carries = reinterpret_cast<float2 *>(carries);
  a.vec = sel_vec(a, time);
  auto kern = sel_fwd_kernel<kSelThreads, kSelK, BF>;
  kern<<<sel_grid(kern, a.rows), kSelThreads, 0, stream>>>(a);
  return launch_status();
}

template <bool BF>
int sel_backward_impl(const float *z, const rqf_selective_inputs *inputs,
                      const rqf_selective_options *options, const float *carries,
                      const float *grad_raw, const float *grad_act, int truncated, float *dz,
                      float *dzw, void *dgamma, void *dwarp, void *dwrite, float *dbias,
                      float *dtheta, void *scratch, int64_t filters, int64_t batch, int64_t time,
                      rqf_stream_t stream) {
  int st = sel_check(z, inputs, options, filters, batch, time);
  if (st != RQF_OK) return st;
  if (filters * batch * time == 0) {
    if (dbias && filters > 0 && cudaMemsetAsync(dbias, 0, filters * sizeof(float), stream))
      return RQF_ERR_LAUNCH;
    if (dtheta && filters > 0 && cudaMemsetAsync(dtheta, 0, filters * sizeof(float), stream))
      return RQF_ERR_LAUNCH;
    return RQF_OK;
  }
  if (!carries || !dz || !dbias || !dtheta || !scratch || (truncated && !dzw) ||
      (options->has_gamma && !dgamma) || (options->has_warp && !dwarp) ||
      (options->has_write && !dwrite))
    return RQF_ERR_ARGUMENT;
  if (!aligned(dz, 8) || (dzw && !aligned(dzw, 8)) || !aligned(carries, 8) ||
      !aligned(scratch, 16) || (grad_raw && !aligned(grad_raw, 8)) ||
      (grad_act && !aligned(grad_act, 8)))
    return RQF_ERR_ALIGN;
  SelArgs a = sel_args(z, inputs, options, filters, batch, time);
  a.carries = const_cast<float2 *>(reinterpret_cast<const float2 *>(carries));
  a.gy = reinterpret_cast<const float2 *>(grad_raw);
  a.gx = reinterpret_cast<const float2 *>(grad_act);
  a.dz = reinterpret_cast<float2 *>(dz);
  a.dzw = reinterpret_cast<float2 *>(dzw);
  a.dG = dgamma;
  a.dW = dwrite;
  a.truncated = truncated ? 1 : 0;
  const size_t dd_bytes =
      options->has_warp ? round256((size_t)filters * batch * time * sizeof(float)) : 0;
  a.dD = options->has_warp ? static_cast<float *>(scratch) : nullptr;
  a.partials = at<float>(scratch, dd_bytes);
  a.vec = sel_vec(a, time);
  auto kern = sel_bwd_kernel<kSelThreads, kSelK, BF>;
  kern<<<sel_grid(kern, a.rows), kSelThreads, 0, stream>>>(a);
  if ((st = launch_status()) != RQF_OK) return st;
  if (options->has_warp) {
    const int64_t bt = batch * time;
    int *order = at<int>(scratch, dd_bytes + round256((size_t)filters * batch * 2 * sizeof(float)));
    int *bounds = order + filters;
    const int ng = (int)inputs->num_groups;
    sel_group_order_kernel<<<1, 32 * ng, 0, stream>>>(a.groups, (int)filters, ng, order, bounds);
    if ((st = launch_status()) != RQF_OK) return st;
    sel_group_reduce_kernel<BF><<<(unsigned)ceil_div(bt, 256), 256, 0, stream>>>(
        a.dD, order, bounds, dwarp, ng, bt);
    if ((st = launch_status()) != RQF_OK) return st;
  }
  sel_param_reduce_kernel<<<(unsigned)ceil_div(filters, 128), 128, 0, stream>>>(
      a.partials, dbias, dtheta, (int)filters, (int)batch);
  return launch_status();
}

}  // namespace

extern "C" {

int rqf_selective_forward(const float *z, const rqf_selective_inputs *inputs,
                          const rqf_selective_options *options, float *raw, float *act,
                          float *carries, int64_t filters, int64_t batch, int64_t time,
                          rqf_stream_t stream) {
  return sel_forward_impl<false>(z, inputs, options, raw, act, carries, filters, batch, time,
                                 stream);
}

int rqf_selective_backward(const float *z, const rqf_selective_inputs *inputs,
                           const rqf_selective_options *options, const float *carries,
                           const float *grad_raw, const float *grad_act, int truncated,
                           float *dz, float *dzw, float *dgamma, float *dwarp, float *dwrite,
                           float *dbias, float *dtheta, void *scratch, int64_t filters,
                           int64_t batch, int64_t time, rqf_stream_t stream) {
  return sel_backward_impl<false>(z, inputs, options, carries, grad_raw, grad_act, truncated, dz,
                                  dzw, dgamma, dwarp, dwrite, dbias, dtheta, scratch, filters,
                                  batch, time, stream);
}

int rqf_selective_forward_bf16(const float *z, const rqf_selective_inputs *inputs,
                               const rqf_selective_options *options, void *raw, void *act,
                               float *carries, int64_t filters, int64_t batch, int64_t time,
                               rqf_stream_t stream) {
  return sel_forward_impl<true>(z, inputs, options, raw, act, carries, filters, batch, time,
                                stream);
}

int rqf_selective_backward_bf16(const float *z, const rqf_selective_inputs *inputs,
                                const rqf_selective_options *options, const float *carries,
                                const float *grad_raw, const float *grad_act, int truncated,
                                float *dz, float *dzw, void *dgamma, void *dwarp, void *dwrite,
                                float *dbias, float *dtheta, void *scratch, int64_t filters,
                                int64_t batch, int64_t time, rqf_stream_t stream) {
  return sel_backward_impl<true>(z, inputs, options, carries, grad_raw, grad_act, truncated, dz,
                                 dzw, dgamma, dwarp, dwrite, dbias, dtheta, scratch, filters,
                                 batch, time, stream);
}

}  // extern "C"

#include "noalloc.cuh"

// ------------------------------------------------ complex projection GEMM
namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D fp32 tensor map: `inner` contiguous elements per row, `outer` rows
// `row_bytes` apart; out-of-range elements load as zero.
bool encode_map_2d(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
                   uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                   CUtensorMapSwizzle swizzle) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = tensor_map_encoder();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t elem[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims, strides, box,
            elem, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct ProjGeometry {
  int64_t rows_pad, k_pad;
};

inline ProjGeometry proj_geometry(int64_t m, int64_t k) {
  ProjGeometry g;
  g.rows_pad = ceil_div(2 * m, proj::kPairM) * proj::kPairM;
  g.k_pad = ceil_div(k, proj::kBK) * proj::kBK;
  return g;
}

// How many CTA pairs (clusters of 2) of `kernel` the device holds at once,
// after raising its dynamic shared-memory limit; 0 on failure.  Cached per
// device and kernel.
template <int kSlot>
int pair_capacity(const void *kernel, int threads, int smem) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  static std::mutex mu;
  static int cached[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return 0;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(sms & ~1), 1, 1);
    cfg.blockDim = dim3((unsigned)threads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sms / 2;  // one CTA per SM, SMs paired per TPC
    }
    cached[dev] = n;
  }
  return cached[dev];
}

int proj_pairs_per_device() {
  return pair_capacity<0>(reinterpret_cast<const void *>(proj::proj_kernel<false>),
                          proj::kThreads, proj::kSmemBytes);
}

}  // namespace

extern "C" {

int rqf_projection_timeout_site(int clear) {
  int site = 0;
  if (cudaMemcpyFromSymbol(&site, proj::g_proj_timeout_site, sizeof(int)) != cudaSuccess) return -1;
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(proj::g_proj_timeout_site, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return site;
}

size_t rqf_projection_workspace_bytes(int64_t m, int64_t k) {
  if (m <= 0 || k <= 0) return 0;
  const ProjGeometry g = proj_geometry(m, k);
  return (size_t)(2 * g.rows_pad * g.k_pad) * sizeof(float);
}

}  // extern "C"

namespace {

int proj_scan_pairs_per_device(int mode) {
  if (mode == proj::kScanBwd)
    return pair_capacity<5>(reinterpret_cast<const void *>(proj::proj_kernel<false, proj::kScanBwd>),
                            proj::kThreads, proj::kScanBwdSmemBytes);
  return pair_capacity<4>(reinterpret_cast<const void *>(proj::proj_kernel<false, proj::kScanFwd>),
                          proj::kThreads, proj::kScanSmemBytes);
}

// x complex (k x n) when real_x = 0, real (k x n) when real_x = 1.  With
// `scan` (complex x, n = batch * T): the block scan (scan_mode kScanFwd, no
// acc) or its VJP (kScanBwd) runs in the epilogue; the caller has checked its
// shapes and zeroed its flags, and chains is filled in here.
int projection_impl(const float *w, const float *x, const float *acc, float *out, int64_t m,
                    int64_t k, int64_t n, int conj_transpose, void *workspace,
                    rqf_stream_t stream, int real_x, const proj::ScanParams *scan = nullptr,
                    int scan_mode = 0) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (m < 0 || k < 0 || n < 0) return RQF_ERR_SHAPE;
  if (m == 0 || n == 0) return RQF_OK;
  if (out == nullptr || (k > 0 && (w == nullptr || x == nullptr || workspace == nullptr)))
    return RQF_ERR_ARGUMENT;
  const size_t out_bytes = (size_t)m * (size_t)n * sizeof(float2);
  if (k == 0) {  // empty sum
    const cudaError_t e = acc ? (acc == out ? cudaSuccess
                                            : cudaMemcpyAsync(out, acc, out_bytes,
                                                              cudaMemcpyDeviceToDevice, st))
                              : cudaMemsetAsync(out, 0, out_bytes, st);
    return e == cudaSuccess ? RQF_OK : RQF_ERR_LAUNCH;
  }
  // TMA: the X' row pitch (8n bytes complex, 4n real) must be a multiple of
  // 16, coordinates are int32.
  if ((n & (real_x ? 3 : 1)) != 0 || n >= (int64_t(1) << 30) || k > 0x7fffffffLL ||
      m > (int64_t(1) << 40))
    return RQF_ERR_SHAPE;
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(workspace, 16) ||
      (acc != nullptr && !aligned(acc, 16)))
    return RQF_ERR_ALIGN;
  const ProjGeometry g = proj_geometry(m, k);
  if (g.rows_pad > 0x3fffffffLL || g.k_pad > 0x7fffffffLL) return RQF_ERR_SHAPE;
  const int pairs = scan ? proj_scan_pairs_per_device(scan_mode) : proj_pairs_per_device();
  if (pairs <= 0) return RQF_ERR_LAUNCH;

  float *a_split = static_cast<float *>(workspace);
  {
    const int64_t total = g.rows_pad * g.k_pad;
    const int64_t blocks = ceil_div(total, 256);
    proj::proj_prep_kernel<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, st>>>(
        reinterpret_cast<const float2 *>(w), a_split, m, (int)k, (int)g.rows_pad, (int)g.k_pad,
        conj_transpose ? 1 : 0);
    if (cudaGetLastError() != cudaSuccess) return RQF_ERR_LAUNCH;
  }
  CUtensorMap tmA, tmX;
  if (!encode_map_2d(&tmA, a_split, (uint64_t)g.k_pad, (uint64_t)(2 * g.rows_pad),
                     (uint64_t)g.k_pad * sizeof(float), proj::kBK, proj::kBM,
                     CU_TENSOR_MAP_SWIZZLE_64B) ||
      !encode_map_2d(&tmX, x, (uint64_t)(real_x ? n : 2 * n), (uint64_t)k,
                     (uint64_t)(real_x ? n : 2 * n) * sizeof(float), 32, proj::kBK,
                     CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
    return RQF_ERR_LAUNCH;

  proj::Params p;
  p.out = reinterpret_cast<float2 *>(out);
  p.acc = reinterpret_cast<const float2 *>(acc);
  p.M = m;
  p.N = n;
  p.K = (int)k;
  p.m_pairs = (int)(g.rows_pad / proj::kPairM);
  p.n_tiles = (int)ceil_div(real_x ? n : 2 * n, proj::kBN);
  p.k_blocks = (int)(g.k_pad / proj::kBK);
  p.num_tiles = (long long)p.m_pairs * p.n_tiles;
  p.a_rows_pad = (int)g.rows_pad;
  p.real_x = real_x;
  const long long grid = 2 * (p.num_tiles < pairs ? p.num_tiles : pairs);  // whole CTA pairs
  p.out_real = nullptr;
  p.scan = scan ? 1 : 0;
  // out == acc (complex x): the epilogue adds into out with TMA reduces
  // instead of loading acc
  p.inplace = (!scan && !real_x && acc != nullptr && acc == out) ? 1 : 0;
  proj::ScanParams plain_sp{};
  if (p.inplace) {
    p.acc = nullptr;
    const uint64_t nf = 2 * (uint64_t)n;
    if (!encode_map_2d(&plain_sp.tmZ, out, nf, (uint64_t)m, nf * sizeof(float), 32, 16,
                       CU_TENSOR_MAP_SWIZZLE_128B))
      return RQF_ERR_LAUNCH;
  }
  if (scan) {
    // Every CTA pair must be resident at once: a tile's epilogue waits for
    // the tile before it along time, which another pair may hold.  The
    // persistent grid is the device's pair capacity at most.
    proj::ScanParams sp = *scan;
    sp.chains = p.m_pairs * sp.batch;
    if (scan_mode == proj::kScanBwd)
      proj::proj_kernel<false, proj::kScanBwd>
          <<<(unsigned)grid, proj::kThreads, proj::kScanBwdSmemBytes, st>>>(tmA, tmX, p, sp);
    else
      proj::proj_kernel<false, proj::kScanFwd>
          <<<(unsigned)grid, proj::kThreads, proj::kScanSmemBytes, st>>>(tmA, tmX, p, sp);
  } else {
    proj::proj_kernel<false><<<(unsigned)grid, proj::kThreads, proj::kSmemBytes, st>>>(
        tmA, tmX, p, plain_sp);
  }
  return launch_status();
}

// Workspace of rqf_projection_block_scan: the split op(W), then the link
// records (num_tiles x 2 ranks x 64 rows of float4), then the flags
// (num_tiles x 8 + 1 abort word).
struct BlockScanLayout {
  size_t link_off, flags_off, flags_bytes, total;
  int64_t num_tiles;
};

bool block_scan_layout(int64_t filters, int64_t k, int64_t batch, int64_t time,
                       BlockScanLayout &l) {
  if (filters <= 0 || k <= 0 || batch <= 0 || time <= 0 || time % 128 != 0) return false;
  if (fbt_dims_ok(filters, batch, time) != RQF_OK || k > 0x7fffffffLL) return false;
  if (batch * time >= (int64_t(1) << 30)) return false;
  const ProjGeometry g = proj_geometry(filters, k);
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  l.num_tiles = (g.rows_pad / proj::kPairM) * (batch * time / 128);
  l.link_off = up((size_t)(2 * g.rows_pad * g.k_pad) * sizeof(float));
  l.flags_off = l.link_off + up((size_t)l.num_tiles * 2 * 64 * sizeof(float4));
  l.flags_bytes = (size_t)(l.num_tiles * 8 + 1) * sizeof(unsigned);
  l.total = l.flags_off + up(l.flags_bytes);
  return true;
}

}  // namespace

extern "C" {

int rqf_projection(const float *w, const float *x, const float *acc, float *out, int64_t m,
                   int64_t k, int64_t n, int conj_transpose, void *workspace,
                   rqf_stream_t stream) {
  return projection_impl(w, x, acc, out, m, k, n, conj_transpose, workspace, stream, 0);
}

int rqf_projection_real(const float *w, const float *x, const float *acc, float *out, int64_t m,
                        int64_t k, int64_t n, int conj_transpose, void *workspace,
                        rqf_stream_t stream) {
  return projection_impl(w, x, acc, out, m, k, n, conj_transpose, workspace, stream, 1);
}

size_t rqf_projection_block_scan_workspace_bytes(int64_t filters, int64_t k, int64_t batch,
                                                 int64_t time) {
  BlockScanLayout l;
  return block_scan_layout(filters, k, batch, time, l) ? l.total : 0;
}

int rqf_projection_block_scan(const float *w, const float *x, const float *c1, const float *tap0,
                              const float *tap1, const float *skip, float *z, float *out,
                              float *carries, void *workspace, int64_t filters, int64_t k,
                              int64_t batch, int64_t time, int fuse_act, rqf_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (k < 0) return RQF_ERR_SHAPE;
  int status = fbt_dims_ok(filters, batch, time);
  if (status != RQF_OK) return status;
  if (filters == 0 || batch == 0 || time == 0) return RQF_OK;
  BlockScanLayout l;
  if (!block_scan_layout(filters, k, batch, time, l)) return RQF_ERR_SHAPE;
  if (!w || !x || !c1 || !tap0 || !tap1 || !z || !out || !carries || !workspace)
    return RQF_ERR_ARGUMENT;
  // out is written while other tiles still read x, z and skip
  if (out == x || out == z || out == skip || z == x || (skip && z == skip))
    return RQF_ERR_ARGUMENT;
  if (!aligned(x, 16) || !aligned(z, 16) || !aligned(out, 16) || !aligned(carries, 16) ||
      !aligned(workspace, 16) || (skip && !aligned(skip, 16)) || !aligned(c1, 8) ||
      !aligned(tap0, 8) || !aligned(tap1, 8))
    return RQF_ERR_ALIGN;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  unsigned *flags = reinterpret_cast<unsigned *>(ws + l.flags_off);
  if (cudaMemsetAsync(flags, 0, l.flags_bytes, st) != cudaSuccess) return RQF_ERR_LAUNCH;
  proj::ScanParams sp{};
  // z and out as (filters rows, 2 batch time floats): the epilogue's TMA
  // stores write 16 rows x 16 complex samples per box
  const uint64_t nf = 2 * (uint64_t)batch * (uint64_t)time;
  if (!encode_map_2d(&sp.tmZ, z, nf, (uint64_t)filters, nf * sizeof(float), 32, 16,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map_2d(&sp.tmAct, out, nf, (uint64_t)filters, nf * sizeof(float), 32, 16,
                     CU_TENSOR_MAP_SWIZZLE_128B))
    return RQF_ERR_LAUNCH;
  sp.c1 = reinterpret_cast<const float2 *>(c1);
  sp.tap0 = reinterpret_cast<const float2 *>(tap0);
  sp.tap1 = reinterpret_cast<const float2 *>(tap1);
  sp.skip = reinterpret_cast<const float2 *>(skip);
  sp.act = reinterpret_cast<float2 *>(out);
  sp.carries = reinterpret_cast<float2 *>(carries);
  sp.link = reinterpret_cast<float4 *>(ws + l.link_off);
  sp.flags = flags;
  sp.T = time;
  sp.batch = (int)batch;
  sp.tiles_per_row = (int)(time / 128);
  sp.fbt_ntiles = (int)rqf_fbt_num_tiles(time);
  sp.fuse_act = fuse_act ? 1 : 0;
  return projection_impl(w, x, nullptr, z, filters, k, batch * time, 0, workspace, stream, 0, &sp,
                         proj::kScanFwd);
}

size_t rqf_projection_block_scan_backward_workspace_bytes(int64_t filters, int64_t k,
                                                          int64_t batch, int64_t time) {
  BlockScanLayout l;
  if (!block_scan_layout(filters, k, batch, time, l)) return 0;
  return l.total + (size_t)filters * (size_t)batch * (size_t)(time / 128) * 3 * sizeof(float2);
}

int rqf_projection_block_scan_backward(const float *w, const float *gz_above, const float *acc,
                                       const float *c1, const float *tap0, const float *tap1,
                                       const float *z, const float *carries, float *grad_out,
                                       float *grad_z, float *grad_c1, float *grad_tap0,
                                       float *grad_tap1, void *workspace, int64_t filters,
                                       int64_t k, int64_t batch, int64_t time, int fuse_act,
                                       rqf_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (k < 0) return RQF_ERR_SHAPE;
  int status = fbt_dims_ok(filters, batch, time);
  if (status != RQF_OK) return status;
  if (filters == 0) return RQF_OK;
  if (batch == 0 || time == 0) {  // empty sums
    const size_t nb = (size_t)filters * sizeof(float2);
    for (float *g : {grad_c1, grad_tap0, grad_tap1})
      if (g && cudaMemsetAsync(g, 0, nb, st) != cudaSuccess) return RQF_ERR_LAUNCH;
    return RQF_OK;
  }
  BlockScanLayout l;
  if (!block_scan_layout(filters, k, batch, time, l)) return RQF_ERR_SHAPE;
  if (!w || !gz_above || !c1 || !tap0 || !tap1 || !z || !carries || !grad_out || !grad_z ||
      !grad_c1 || !grad_tap0 || !grad_tap1 || !workspace)
    return RQF_ERR_ARGUMENT;
  // the outputs are written while other tiles still read gz_above, acc and z
  for (const float *in : {gz_above, acc, z, carries})
    if (in && (in == grad_out || in == grad_z)) return RQF_ERR_ARGUMENT;
  if (grad_out == grad_z) return RQF_ERR_ARGUMENT;
  if (!aligned(gz_above, 16) || !aligned(z, 16) || !aligned(grad_out, 16) ||
      !aligned(grad_z, 16) || !aligned(carries, 16) || !aligned(workspace, 16) ||
      (acc && !aligned(acc, 16)) || !aligned(c1, 8) || !aligned(tap0, 8) || !aligned(tap1, 8) ||
      !aligned(grad_c1, 8) || !aligned(grad_tap0, 8) || !aligned(grad_tap1, 8))
    return RQF_ERR_ALIGN;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  unsigned *flags = reinterpret_cast<unsigned *>(ws + l.flags_off);
  float2 *partials = reinterpret_cast<float2 *>(ws + l.total);
  if (cudaMemsetAsync(flags, 0, l.flags_bytes, st) != cudaSuccess) return RQF_ERR_LAUNCH;
  proj::ScanParams sp{};
  const uint64_t nf = 2 * (uint64_t)batch * (uint64_t)time;
  if (!encode_map_2d(&sp.tmZ, grad_out, nf, (uint64_t)filters, nf * sizeof(float), 32, 16,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map_2d(&sp.tmAct, grad_z, nf, (uint64_t)filters, nf * sizeof(float), 32, 16,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map_2d(&sp.tmZin, z, nf, (uint64_t)filters, nf * sizeof(float), 32, 16,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
      (acc && !encode_map_2d(&sp.tmAcc, acc, nf, (uint64_t)filters, nf * sizeof(float), 32, 16,
                             CU_TENSOR_MAP_SWIZZLE_128B)))
    return RQF_ERR_LAUNCH;
  sp.c1 = reinterpret_cast<const float2 *>(c1);
  sp.tap0 = reinterpret_cast<const float2 *>(tap0);
  sp.tap1 = reinterpret_cast<const float2 *>(tap1);
  sp.carries = const_cast<float2 *>(reinterpret_cast<const float2 *>(carries));  // read only
  sp.zin = reinterpret_cast<const float2 *>(z);
  sp.partials = partials;
  sp.reverse = 1;
  sp.link = reinterpret_cast<float4 *>(ws + l.link_off);
  sp.flags = flags;
  sp.T = time;
  sp.batch = (int)batch;
  sp.tiles_per_row = (int)(time / 128);
  sp.fbt_ntiles = (int)rqf_fbt_num_tiles(time);
  sp.fuse_act = fuse_act ? 1 : 0;
  status = projection_impl(w, gz_above, acc, grad_out, filters, k, batch * time, 1, workspace,
                           stream, 0, &sp, proj::kScanBwd);
  if (status != RQF_OK) return status;
  reduce_partials_kernel<<<(unsigned)filters, 256, 0, st>>>(
      partials, reinterpret_cast<float2 *>(grad_c1), reinterpret_cast<float2 *>(grad_tap0),
      reinterpret_cast<float2 *>(grad_tap1), batch, batch, 1, sp.tiles_per_row);
  return launch_status();
}

size_t rqf_projection_real_out_workspace_bytes(int64_t m, int64_t k) {
  if (m <= 0 || k <= 0) return 0;
  const int64_t rows_pad = ceil_div(m, proj::kPairM) * proj::kPairM;
  const int64_t k3_pad = ceil_div(k, proj::kBK / 2) * proj::kBK;
  return (size_t)(2 * rows_pad * k3_pad) * sizeof(float);
}

int rqf_projection_real_out(const float *w, const float *x, float *out, int64_t m, int64_t k,
                            int64_t n, void *workspace, rqf_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (m < 0 || k < 0 || n < 0) return RQF_ERR_SHAPE;
  if (m == 0 || n == 0) return RQF_OK;
  if (out == nullptr || (k > 0 && (w == nullptr || x == nullptr || workspace == nullptr)))
    return RQF_ERR_ARGUMENT;
  if (k == 0)
    return cudaMemsetAsync(out, 0, (size_t)m * (size_t)n * sizeof(float), st) == cudaSuccess
               ? RQF_OK
               : RQF_ERR_LAUNCH;
  // float4 output stores and the x row pitch (8n bytes): n a multiple of 4
  if ((n & 3) != 0 || n >= (int64_t(1) << 30) || k > 0x7fffffffLL || m > (int64_t(1) << 40))
    return RQF_ERR_SHAPE;
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(workspace, 16)) return RQF_ERR_ALIGN;
  const int64_t rows_pad = ceil_div(m, proj::kPairM) * proj::kPairM;
  const int64_t kblocks = ceil_div(k, proj::kBK / 2);
  const int64_t k3_pad = kblocks * proj::kBK;
  if (rows_pad > 0x3fffffffLL || k3_pad > 0x7fffffffLL) return RQF_ERR_SHAPE;
  const int pairs = pair_capacity<3>(reinterpret_cast<const void *>(proj::proj_kernel<true>),
                                     proj::kThreads, proj::ProjLayout<true>::kSmemBytes);
  if (pairs <= 0) return RQF_ERR_LAUNCH;
  float *a_split = static_cast<float *>(workspace);
  {
    const int64_t total = rows_pad * k3_pad;
    const int64_t blocks = ceil_div(total, 256);
    proj::proj_prep_real_out_kernel<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, st>>>(
        reinterpret_cast<const float2 *>(w), a_split, m, (int)k, (int)rows_pad, (int)k3_pad);
    if (cudaGetLastError() != cudaSuccess) return RQF_ERR_LAUNCH;
  }
  CUtensorMap tmA, tmX;
  if (!encode_map_2d(&tmA, a_split, (uint64_t)k3_pad, (uint64_t)(2 * rows_pad),
                     (uint64_t)k3_pad * sizeof(float), proj::kBK, proj::kBM,
                     CU_TENSOR_MAP_SWIZZLE_64B) ||
      !encode_map_2d(&tmX, x, (uint64_t)(2 * n), (uint64_t)k, (uint64_t)(2 * n) * sizeof(float),
                     2 * proj::kBNh, proj::kBK / 2, CU_TENSOR_MAP_SWIZZLE_NONE))
    return RQF_ERR_LAUNCH;
  proj::Params p;
  p.out = nullptr;
  p.acc = nullptr;
  p.out_real = out;
  p.M = m;
  p.N = n;
  p.K = (int)k;
  p.m_pairs = (int)(rows_pad / proj::kPairM);
  p.n_tiles = (int)ceil_div(n, proj::kBN);
  p.k_blocks = (int)kblocks;
  p.num_tiles = (long long)p.m_pairs * p.n_tiles;
  p.a_rows_pad = (int)rows_pad;
  p.real_x = 0;
  const long long grid = 2 * (p.num_tiles < pairs ? p.num_tiles : pairs);
  p.scan = 0;
  p.inplace = 0;
  proj::proj_kernel<true><<<(unsigned)grid, proj::kThreads, proj::ProjLayout<true>::kSmemBytes,
                            st>>>(tmA, tmX, p, proj::ScanParams{});
  return launch_status();
}

}  // extern "C"

// ------------------------------------------------ projection weight gradient
namespace {

struct WgGeometry {
  int m_pairs, i_tiles, splits;
  int64_t kblocks;
};

// kblocks: k-blocks of the reduction, ceil(2n / 16) for complex gz and
// ceil(n / 16) for real gz.
inline WgGeometry wgrad_geometry(int64_t m, int64_t k, int64_t kblocks, int pairs) {
  WgGeometry g;
  g.m_pairs = (int)ceil_div(m, proj::kWgPairRows);
  g.i_tiles = (int)ceil_div(k, proj::kWgCols);
  g.kblocks = kblocks;
  const int64_t tiles = (int64_t)g.m_pairs * g.i_tiles;
  // whole waves of CTA pairs (one CTA per SM), enough of them that no pair
  // runs more than ~256 k-blocks: pairs sharing an operand block then stay
  // close enough in progress for the block's second read to hit L2
  int64_t per_wave = pairs > 0 ? pairs / tiles : 1;
  if (per_wave < 1) per_wave = 1;
  int64_t waves = ceil_div(g.kblocks, per_wave * 256);
  if (waves > 16) waves = 16;
  if (waves < 1) waves = 1;
  int64_t splits = per_wave * waves;
  if (splits > g.kblocks) splits = g.kblocks;
  g.splits = (int)splits;
  return g;
}

template <bool kRealGz>
int wgrad_pairs_per_device() {
  return pair_capacity<kRealGz ? 2 : 1>(
      reinterpret_cast<const void *>(proj::proj_wgrad_kernel<kRealGz>), proj::kWgThreads,
      proj::WgLayout<kRealGz>::kSmemBytes);
}

inline int64_t wgrad_kblocks(int64_t n, bool real_gz) {
  return real_gz ? ceil_div(n, proj::WgLayout<true>::kBKw)
                 : ceil_div(2 * n, proj::WgLayout<false>::kBKw);
}

template <bool kRealGz>
size_t wgrad_workspace_bytes(int64_t m, int64_t k, int64_t n) {
  if (m <= 0 || k <= 0 || n <= 0) return 0;
  const WgGeometry g =
      wgrad_geometry(m, k, wgrad_kblocks(n, kRealGz), wgrad_pairs_per_device<kRealGz>());
  return (size_t)g.splits * (size_t)g.m_pairs * proj::kWgPairRows * (size_t)g.i_tiles *
         proj::kWgCols * sizeof(float2);
}

// gz complex (m x n) or, with kRealGz, real (m x n); x complex (k x n).
template <bool kRealGz>
int wgrad_impl(const float *gz, const float *x, float *gw, int64_t m, int64_t k, int64_t n,
               void *workspace, rqf_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (m < 0 || k < 0 || n < 0) return RQF_ERR_SHAPE;
  if (m == 0 || k == 0) return RQF_OK;
  if (gw == nullptr) return RQF_ERR_ARGUMENT;
  if (n == 0) {
    return cudaMemsetAsync(gw, 0, (size_t)m * (size_t)k * sizeof(float2), st) == cudaSuccess
               ? RQF_OK
               : RQF_ERR_LAUNCH;
  }
  if (gz == nullptr || x == nullptr || workspace == nullptr) return RQF_ERR_ARGUMENT;
  // TMA row pitches (8n bytes complex, 4n real) must be multiples of 16.
  if ((n & (kRealGz ? 3 : 1)) != 0 || n >= (int64_t(1) << 30) || m > 0x7fffffffLL ||
      k > 0x7fffffffLL)
    return RQF_ERR_SHAPE;
  if (!aligned(gz, 16) || !aligned(x, 16) || !aligned(workspace, 16)) return RQF_ERR_ALIGN;
  const int pairs = wgrad_pairs_per_device<kRealGz>();
  if (pairs <= 0) return RQF_ERR_LAUNCH;
  const WgGeometry g = wgrad_geometry(m, k, wgrad_kblocks(n, kRealGz), pairs);
  const uint64_t gz_cols = kRealGz ? (uint64_t)n : (uint64_t)(2 * n);
  CUtensorMap tmG, tmH;
  // boxes of 32 floats x rows, 128-byte swizzle: gz' and h' (complex gz), or
  // g (32 samples) and h' (two boxes per stage: 32 samples as (Re, Im) pairs,
  // de-interleaved in shared memory) for real gz
  constexpr int bk = proj::WgLayout<kRealGz>::kBKw;
  const bool ok_g = encode_map_2d(&tmG, gz, gz_cols, (uint64_t)m, gz_cols * sizeof(float), bk,
                                  proj::kWgRows, CU_TENSOR_MAP_SWIZZLE_128B);
  const bool ok_h = encode_map_2d(&tmH, x, (uint64_t)(2 * n), (uint64_t)k,
                                  (uint64_t)(2 * n) * sizeof(float), bk, proj::kWgHRows,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
  if (!ok_g || !ok_h) return RQF_ERR_LAUNCH;
  proj::WgParams p;
  p.partials = static_cast<float2 *>(workspace);
  p.M = m;
  p.K = k;
  p.m_pairs = g.m_pairs;
  p.i_tiles = g.i_tiles;
  p.splits = g.splits;
  p.kblocks = g.kblocks;
  p.ld = g.i_tiles * proj::kWgCols;
  const int64_t grid = 2 * (int64_t)g.m_pairs * g.i_tiles * g.splits;  // whole CTA pairs
  proj::proj_wgrad_kernel<kRealGz>
      <<<(unsigned)grid, proj::kWgThreads, proj::WgLayout<kRealGz>::kSmemBytes, st>>>(tmG, tmH, p);
  if (cudaGetLastError() != cudaSuccess) return RQF_ERR_LAUNCH;
  const int64_t total = m * k;
  const int64_t blocks = ceil_div(total, 32);
  if (blocks > 0x7fffffffLL) return RQF_ERR_SHAPE;
  proj::proj_wgrad_reduce_kernel<<<(unsigned)blocks, 32 * proj::kWgReduceGroups, 0, st>>>(
      p.partials, reinterpret_cast<float2 *>(gw), m, k, g.splits,
      (long long)g.m_pairs * proj::kWgPairRows, p.ld);
  return launch_status();
}

}  // namespace

extern "C" {

size_t rqf_projection_weight_grad_workspace_bytes(int64_t m, int64_t k, int64_t n) {
  return wgrad_workspace_bytes<false>(m, k, n);
}

int rqf_projection_weight_grad(const float *gz, const float *x, float *gw, int64_t m, int64_t k,
                               int64_t n, void *workspace, rqf_stream_t stream) {
  return wgrad_impl<false>(gz, x, gw, m, k, n, workspace, stream);
}

size_t rqf_projection_weight_grad_real_workspace_bytes(int64_t m, int64_t k, int64_t n) {
  return wgrad_workspace_bytes<true>(m, k, n);
}

int rqf_projection_weight_grad_real(const float *gz, const float *x, float *gw, int64_t m,
                                    int64_t k, int64_t n, void *workspace, rqf_stream_t stream) {
  return wgrad_impl<true>(gz, x, gw, m, k, n, workspace, stream);
}

}  // extern "C"

// ------------------------------------------------ low-rank first block
extern "C" {

int rqf_lowrank_drive(const float *u, const float *beta, const float *w_in, const float *b_in,
                      const float *x, float *z, float *h, int64_t f, int64_t n, int i,
                      rqf_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (f < 0 || n < 0 || i < 0 || i > lowrank::kMaxRank) return RQF_ERR_SHAPE;
  if (f == 0 || n == 0) return RQF_OK;
  if ((n & 1) != 0) return RQF_ERR_SHAPE;
  if (z == nullptr || (i > 0 && (u == nullptr || x == nullptr)) ||
      (h != nullptr && i > 0 && w_in == nullptr))
    return RQF_ERR_ARGUMENT;
  if (!aligned(z, 16) || (h != nullptr && !aligned(h, 16)) || (x != nullptr && !aligned(x, 8)))
    return RQF_ERR_ALIGN;
  const int64_t total = f * (n / 2);
  const int64_t blocks = ceil_div(total, 256);
  lowrank::lowrank_drive_kernel<<<(unsigned)(blocks < 8192 ? blocks : 8192), 256, 0, st>>>(
      reinterpret_cast<const float2 *>(u), reinterpret_cast<const float2 *>(beta), w_in, b_in, x,
      reinterpret_cast<float2 *>(z), reinterpret_cast<float2 *>(h), f, n, i);
  return launch_status();
}

size_t rqf_rowdot_workspace_bytes(int64_t f, int64_t n, int i, int with_sum) {
  if (f <= 0 || n <= 0 || i < 0) return 0;
  const int64_t chunks = ceil_div(n, lowrank::kRowdotChunk);
  return (size_t)(f * chunks * (i + (with_sum ? 1 : 0))) * sizeof(double2);
}

int rqf_rowdot(const float *a, const float *x, float *out, void *workspace, int64_t f, int64_t n,
               int i, int with_sum, rqf_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int J = i + (with_sum ? 1 : 0);
  if (f < 0 || n < 0 || i < 0 || i > lowrank::kMaxRank || f > 65535) return RQF_ERR_SHAPE;
  if (f == 0 || J == 0) return RQF_OK;
  if (out == nullptr) return RQF_ERR_ARGUMENT;
  if (n == 0)
    return cudaMemsetAsync(out, 0, (size_t)(f * J) * sizeof(float2), st) == cudaSuccess
               ? RQF_OK
               : RQF_ERR_LAUNCH;
  if ((n & 1) != 0) return RQF_ERR_SHAPE;
  if (a == nullptr || workspace == nullptr || (i > 0 && x == nullptr)) return RQF_ERR_ARGUMENT;
  if (!aligned(a, 16) || !aligned(workspace, 16) || (x != nullptr && !aligned(x, 8)))
    return RQF_ERR_ALIGN;
  const int64_t chunks = ceil_div(n, lowrank::kRowdotChunk);
  if (chunks > 0x7fffffffLL) return RQF_ERR_SHAPE;
  double2 *partials = static_cast<double2 *>(workspace);
  lowrank::rowdot_partial_kernel<<<dim3((unsigned)chunks, (unsigned)f), lowrank::kRowdotThreads, 0,
                                   st>>>(reinterpret_cast<const float2 *>(a), x, partials, n, i,
                                         with_sum ? 1 : 0, (int)chunks);
  if (cudaGetLastError() != cudaSuccess) return RQF_ERR_LAUNCH;
  const int64_t outs = f * J;
  lowrank::rowdot_finish_kernel<<<(unsigned)ceil_div(outs, 256), 256, 0, st>>>(
      partials, reinterpret_cast<float2 *>(out), f, J, (int)chunks);
  return launch_status();
}

}  // extern "C"

// ------------------------------------------------ mean-pooled readout hidden layer
extern "C" {

int rqf_readout_relu_pool(const float *z, const float *bias, uint32_t *mask, float *pooled,
                          int64_t h, int64_t batch, int64_t time, rqf_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (h < 0 || batch < 0 || time < 0) return RQF_ERR_SHAPE;
  const int64_t rows = h * batch;
  if (rows == 0) return RQF_OK;
  if (rows > 0x7fffffffLL || batch > 0x7fffffffLL) return RQF_ERR_SHAPE;
  if (time == 0) return RQF_ERR_SHAPE;  // the mean over no samples is undefined
  if (z == nullptr || mask == nullptr || pooled == nullptr) return RQF_ERR_ARGUMENT;
  readout::relu_pool_kernel<<<(unsigned)rows, readout::kThreads, 0, st>>>(
      z, bias, mask, pooled, (int)batch, time,
      ceil_div(time, 32));
  return launch_status();
}

int rqf_readout_relu_pool_backward(const uint32_t *mask, const float *scale, float *gc,
                                   float *counts, int64_t h, int64_t batch, int64_t time,
                                   rqf_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (h < 0 || batch < 0 || time < 0) return RQF_ERR_SHAPE;
  const int64_t rows = h * batch;
  if (rows == 0 || time == 0) return RQF_OK;
  if (rows > 0x7fffffffLL) return RQF_ERR_SHAPE;
  if (mask == nullptr || scale == nullptr || gc == nullptr) return RQF_ERR_ARGUMENT;
  readout::relu_pool_backward_kernel<<<(unsigned)rows, readout::kThreads, 0, st>>>(
      mask, scale, gc, counts, time, ceil_div(time, 32));
  return launch_status();
}

int rqf_readout_bias_relu(float *z, const float *bias, uint32_t *mask, int64_t h, int64_t batch,
                          int64_t time, rqf_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (h < 0 || batch < 0 || time < 0) return RQF_ERR_SHAPE;
  const int64_t rows = h * batch;
  if (rows == 0 || time == 0) return RQF_OK;
  if (rows > 0x7fffffffLL || batch > 0x7fffffffLL) return RQF_ERR_SHAPE;
  if (z == nullptr || mask == nullptr) return RQF_ERR_ARGUMENT;
  readout::bias_relu_kernel<<<(unsigned)rows, readout::kThreads, 0, st>>>(
      z, bias, mask, (int)batch, time, ceil_div(time, 32));
  return launch_status();
}

int rqf_readout_bias_relu_backward(const float *gy, const uint32_t *mask, float *g, float *rowsum,
                                   int64_t h, int64_t batch, int64_t time, rqf_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (h < 0 || batch < 0 || time < 0) return RQF_ERR_SHAPE;
  const int64_t rows = h * batch;
  if (rows == 0) return RQF_OK;
  if (rows > 0x7fffffffLL) return RQF_ERR_SHAPE;
  if (time == 0) {
    if (rowsum == nullptr) return RQF_OK;
    return cudaMemsetAsync(rowsum, 0, (size_t)rows * sizeof(float), st) == cudaSuccess
               ? RQF_OK
               : RQF_ERR_LAUNCH;
  }
  if (gy == nullptr || mask == nullptr || g == nullptr) return RQF_ERR_ARGUMENT;
  readout::bias_relu_backward_kernel<<<(unsigned)rows, readout::kThreads, 0, st>>>(
      gy, mask, g, rowsum, time, ceil_div(time, 32));
  return launch_status();
}

namespace {
int ce_dims_ok(int64_t classes, int64_t batch, int64_t time) {
  if (classes <= 0 || batch < 0 || time < 0 || classes > 0x7fffffffLL) return RQF_ERR_SHAPE;
  if (ceil_div(batch * time, readout::kCeThreads) > 0x7fffffffLL) return RQF_ERR_SHAPE;
  return RQF_OK;
}
}  // namespace

size_t rqf_per_step_cross_entropy_scratch_bytes(int64_t batch, int64_t time) {
  if (batch <= 0 || time <= 0) return 0;
  return round256((size_t)ceil_div(batch * time, readout::kCeThreads) * sizeof(double));
}

int rqf_per_step_cross_entropy(const float *logits, const int64_t *labels, float *loss,
                               void *scratch, int64_t classes, int64_t batch, int64_t time,
                               float label_smoothing, rqf_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc = ce_dims_ok(classes, batch, time);
  if (rc != RQF_OK) return rc;
  if (loss == nullptr) return RQF_ERR_ARGUMENT;
  const int64_t n = batch * time;
  if (n == 0)  // the mean over no samples, as torch gives it
    return cudaMemsetAsync(loss, 0xff, sizeof(float), st) == cudaSuccess ? RQF_OK : RQF_ERR_LAUNCH;
  if (logits == nullptr || labels == nullptr || scratch == nullptr) return RQF_ERR_ARGUMENT;
  if (!aligned(scratch, 8)) return RQF_ERR_ALIGN;
  const int64_t blocks = ceil_div(n, readout::kCeThreads);
  readout::ce_forward_kernel<<<(unsigned)blocks, readout::kCeThreads, 0, st>>>(
      logits, reinterpret_cast<const long long *>(labels), n, time, (int)classes,
      label_smoothing, static_cast<double *>(scratch));
  if ((rc = launch_status()) != RQF_OK) return rc;
  readout::ce_finalize_kernel<<<1, 32, 0, st>>>(static_cast<const double *>(scratch), blocks, n,
                                                loss);
  return launch_status();
}

int rqf_per_step_cross_entropy_backward(const float *logits, const int64_t *labels,
                                        const float *grad_loss, float *grad_logits,
                                        int64_t classes, int64_t batch, int64_t time,
                                        float label_smoothing, rqf_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc = ce_dims_ok(classes, batch, time);
  if (rc != RQF_OK) return rc;
  const int64_t n = batch * time;
  if (n == 0) return RQF_OK;
  if (logits == nullptr || labels == nullptr || grad_loss == nullptr || grad_logits == nullptr)
    return RQF_ERR_ARGUMENT;
  readout::ce_backward_kernel<<<(unsigned)ceil_div(n, readout::kCeThreads), readout::kCeThreads, 0,
                                st>>>(logits, reinterpret_cast<const long long *>(labels),
                                      grad_loss, n, time, (int)classes, label_smoothing,
                                      grad_logits);
  return launch_status();
}

}  // extern "C"

// ------------------------------------------------ two-tap coefficient producer
extern "C" {

namespace {
int coeff_setup(const rqf_coeff_leaves *leaves, const rqf_coeff_options *opts, int64_t n,
                coef::Leaves *L, coef::Opts *o) {
  if (!leaves || !opts || n < 0) return RQF_ERR_ARGUMENT;
  const int disc = opts->discretization;
  if (disc != RQF_DISC_EULER && disc != RQF_DISC_ZOH && disc != RQF_DISC_FOH)
    return RQF_ERR_ARGUMENT;
  if (!opts->prospective && disc != RQF_DISC_FOH) return RQF_ERR_ARGUMENT;  // single-tap forms
  if (opts->param_space != 0 && opts->param_space != 1) return RQF_ERR_ARGUMENT;
  if (!(opts->dt > 0.0)) return RQF_ERR_ARGUMENT;
  if (!leaves->log_tau && !(opts->tau > 0.0)) return RQF_ERR_ARGUMENT;
  if (n > 0 && (!leaves->theta_leaf || !leaves->gamma_leaf)) return RQF_ERR_ARGUMENT;
  if (n > 0 && opts->param_space == 1 &&
      (!leaves->min_gamma || !leaves->max_gamma || !leaves->min_freq || !leaves->max_freq))
    return RQF_ERR_ARGUMENT;
  *L = {leaves->theta_leaf, leaves->gamma_leaf, leaves->log_tau, leaves->min_gamma,
        leaves->max_gamma, leaves->min_freq, leaves->max_freq, leaves->prospective_tau};
  *o = {disc, opts->prospective ? 1 : 0, opts->gamma_mode ? 1 : 0, opts->param_space,
        opts->clamp_gamma ? 1 : 0, opts->dt, opts->tau};
  return RQF_OK;
}
}  // namespace

int rqf_filter_two_tap_coefficients(const rqf_coeff_leaves *leaves, const rqf_coeff_options *opts,
                                    float *c1, float *tap0, float *tap1, int64_t n,
                                    rqf_stream_t stream) {
  coef::Leaves L;
  coef::Opts o;
  const int rc = coeff_setup(leaves, opts, n, &L, &o);
  if (rc != RQF_OK) return rc;
  if (n == 0) return RQF_OK;
  if (!c1 || !tap0 || !tap1) return RQF_ERR_ARGUMENT;
  if (!aligned(c1, 8) || !aligned(tap0, 8) || !aligned(tap1, 8)) return RQF_ERR_ALIGN;
  coef::two_tap_kernel<<<(unsigned)ceil_div(n, 256), 256, 0,
                         reinterpret_cast<cudaStream_t>(stream)>>>(
      L, o, reinterpret_cast<float2 *>(c1), reinterpret_cast<float2 *>(tap0),
      reinterpret_cast<float2 *>(tap1), n);
  return launch_status();
}

int rqf_filter_two_tap_coefficients_backward(const rqf_coeff_leaves *leaves,
                                             const rqf_coeff_options *opts, const float *grad_c1,
                                             const float *grad_tap0, const float *grad_tap1,
                                             float *grad_theta_leaf, float *grad_gamma_leaf,
                                             float *grad_log_tau, float *grad_prospective_tau,
                                             int64_t n, rqf_stream_t stream) {
  coef::Leaves L;
  coef::Opts o;
  const int rc = coeff_setup(leaves, opts, n, &L, &o);
  if (rc != RQF_OK) return rc;
  if (n == 0) return RQF_OK;
  if (grad_log_tau && !leaves->log_tau) return RQF_ERR_ARGUMENT;
  if (grad_prospective_tau && !leaves->prospective_tau) return RQF_ERR_ARGUMENT;
  if ((grad_c1 && !aligned(grad_c1, 8)) || (grad_tap0 && !aligned(grad_tap0, 8)) ||
      (grad_tap1 && !aligned(grad_tap1, 8)))
    return RQF_ERR_ALIGN;
  if (!grad_theta_leaf && !grad_gamma_leaf && !grad_log_tau && !grad_prospective_tau)
    return RQF_OK;
  coef::two_tap_backward_kernel<<<(unsigned)ceil_div(n, 128), 128, 0,
                                  reinterpret_cast<cudaStream_t>(stream)>>>(
      L, o, reinterpret_cast<const float2 *>(grad_c1), reinterpret_cast<const float2 *>(grad_tap0),
      reinterpret_cast<const float2 *>(grad_tap1), grad_theta_leaf, grad_gamma_leaf, grad_log_tau,
      grad_prospective_tau, n);
  return launch_status();
}

// The log-space ZOH tau-mode form with a scalar tau: the general producer
// with those options.
int rqf_two_tap_coefficients(const float *log_theta, const float *log_gamma, float *c1, float *tap0,
                             float *tap1, int64_t n, double dt, double tau, rqf_stream_t stream) {
  if (n < 0 || !(tau > 0.0) || !(dt > 0.0)) return RQF_ERR_ARGUMENT;
  const rqf_coeff_leaves L = {log_theta, log_gamma, nullptr, nullptr,
                              nullptr,   nullptr,   nullptr, nullptr};
  const rqf_coeff_options o = {RQF_DISC_ZOH, 1, 0, 0, 0, dt, tau};
  return rqf_filter_two_tap_coefficients(&L, &o, c1, tap0, tap1, n, stream);
}

int rqf_two_tap_coefficients_backward(const float *log_theta, const float *log_gamma,
                                      const float *grad_c1, const float *grad_tap0,
                                      const float *grad_tap1, float *grad_log_theta,
                                      float *grad_log_gamma, int64_t n, double dt, double tau,
                                      rqf_stream_t stream) {
  if (n < 0 || !(tau > 0.0) || !(dt > 0.0)) return RQF_ERR_ARGUMENT;
  if (n > 0 && (!grad_log_theta || !grad_log_gamma)) return RQF_ERR_ARGUMENT;
  const rqf_coeff_leaves L = {log_theta, log_gamma, nullptr, nullptr,
                              nullptr,   nullptr,   nullptr, nullptr};
  const rqf_coeff_options o = {RQF_DISC_ZOH, 1, 0, 0, 0, dt, tau};
  return rqf_filter_two_tap_coefficients_backward(&L, &o, grad_c1, grad_tap0, grad_tap1,
                                                  grad_log_theta, grad_log_gamma, nullptr,
                                                  nullptr, n, stream);
}

}  // extern "C"
