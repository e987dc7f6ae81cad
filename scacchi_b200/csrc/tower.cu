// AZDirichletNet leaf evaluation on B200 (network.py:338-524 of the reference,
// resnet_v2, binary outcomes, direct log-concentration heads).
//
// Activation layout ("padded flat"): every board is 100 rows of 128 bf16
// channels, row = y' * 10 + x' with y' = y + 1 in [0, 10) and x' = x in
// [0, 10).  Row y' = 0 and column x' = 9 are zero; they are the SAME
// padding of this board and of its neighbours (the row above board e + 1
// is board e's last zero row; the column left of x = 0 is the previous
// row's zero column).  A 3x3 tap (dy, dx) is then a plain row shift by
// dy * 10 + dx, so the convolution is a GEMM whose A operand for tap t is a
// row-shifted TMA load of the activation matrix (implicit GEMM):
//
//   out[r, n] = sum_t sum_c act[r + off_t, c] * W[t, n, c],  K = 9 * 128.
//
// conv_tc_kernel: persistent (one CTA per SM), warp-specialised, over tile
// pairs of 256 rows.  The nine taps of a pair read overlapping row ranges,
// so A is loaded once per pair and 64-channel half as a 288-row window
// (shared memory traffic per pair: 72 KB of A instead of 18 x 32 KB), and
// each weight tile feeds both 128-row accumulators of the pair.
//   warp 0      TMA producer of the weights: the nine (tap, h) tiles (128
//               out x 64 in) per half through a 4-stage ring
//   warp 10     TMA producer of the windows: half h of the next pair loads
//               as soon as the MMAs finish reading half h of this one
//   warp 1      TMEM allocator and MMA issuer (one thread):
//               tcgen05.mma.cta_group::1.kind::f16, K = 16, 16-bit
//               operands -> fp32 in TMEM.  Every layer runs transposed:
//               M = 128 output channels (A = the weight tile), N = 256 rows
//               of the pair (B = the window from row 16 + shift; any row:
//               the swizzle phase follows the address), so TMEM lane =
//               channel and column = row, and a pair takes half the MMA
//               instructions of two M = N = 128 products (the issue rate of
//               those bounded the kernel).  Two 256-column accumulators, so
//               a pair's epilogue overlaps the next pair
//   warps 2-9   epilogue, two warps per TMEM lane quadrant: fused bias /
//               folded BatchNorm / ReLU / residual / next block's BN-ReLU,
//               bf16 into 128B-swizzled shared memory, TMA store.  They
//               read TMEM with tcgen05.ld 16x256b (the mma fragment
//               layout) and transpose 8x8 blocks into the row-major
//               staging tile with stmatrix .trans; the residual comes back
//               the same way through ldmatrix .trans, and is prefetched
//               into L2 once the CTA's previous pair is done.  The last
//               layer computes the heads'
//               1x1 convolutions from the same fragments: per-thread sums
//               over its channels, a lane butterfly, then the four lane
//               quadrants' partials added in order through shared memory.
//
// Every mbarrier wait is bounded: on timeout the kernel raises an error
// flag, stops issuing, drains its own copies and releases TMEM.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "../../include/scacchi_b200.h"

namespace {

constexpr int kC = 128;          // channels
constexpr int kRowsPerBoard = 100;
constexpr int kBM = 128;         // rows per accumulator tile
constexpr int kBK = 64;          // channels per K block (128 bytes of 16-bit values)
constexpr int kTileBytes = kBM * kBK * 2;  // 16 KB
constexpr int kBStages = 4;      // weight tiles in flight when both staging tiles are in use
constexpr int kMaxBStages = 8;   // ... and when the epilogue leaves staging space unused
constexpr int kBTileBytes = kC * kBK * 2;  // 16 KB: 128 outputs x 64 inputs of one tap
constexpr int kWinLead = 16;     // window rows above (and below) a tile pair: taps shift by <= 11
constexpr int kWinRows = 2 * kBM + 2 * kWinLead;    // 288
constexpr int kWinBoxRows = kWinRows / 2;           // 144 rows per TMA box (<= 256)
constexpr int kWinHalfBytes = kWinRows * kBK * 2;   // 36 KB per 64-channel half
constexpr int kTmemCols = 512;   // two pairs of 128-column accumulators
constexpr int kEpiWarps = 8;     // two per TMEM lane quadrant, 64 columns each
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 64 + kEpiThreads + 32;  // + the window producer warp
constexpr int kHeadCh = 6;       // policy 2, value 1, q mean 2, q concentration 1
constexpr uint32_t kWaitLimit = 1u << 30;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s

__device__ uint32_t g_tower_error;

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .b64 state;\n\t"
      "mbarrier.arrive.shared::cta.b64 state, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: gives up after kWaitNs of wall time (or when another role
// aborted), raising the error flag; returns whether the phase completed.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  for (uint32_t i = 1; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0u) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - start > kWaitNs) break;
    }
  }
  atomicOr(&g_tower_error, 1u);
  *abort_flag = 1;
  return false;
}

// drain wait used while exiting: bounded by time only
__device__ __forceinline__ void mbar_drain(uint64_t *bar, uint32_t parity) {
  const uint64_t start = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - start > kWaitNs) break;
}

__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *smem_src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// bring `bytes` (a multiple of 16) of global memory at a 16-byte aligned
// address into L2 ahead of use
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16, both K-major
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 16 TMEM lanes x 8 columns in the mma fragment layout: thread t receives
// lane t/4 columns 2(t%4), 2(t%4)+1 (r[0], r[1]) and lane t/4 + 8, same
// columns (r[2], r[3]).  Asynchronous until tmem_wait_ld().
__device__ __forceinline__ void tmem_ld16x256(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x1.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// four 8x8 16-bit matrices between the fragment layout (thread t: row t/4,
// columns 2(t%4), 2(t%4)+1 of matrix i in register i) and shared memory,
// transposed: fragment column c is memory row c, whose 16-byte address
// thread 8i + c supplies
__device__ __forceinline__ void stmatrix_x4_trans(uint32_t addr, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (leading offset unused for swizzled K-major layouts).  A
// matrix may start at any 128-byte row of a 1024-byte-aligned swizzled
// tile with the base-offset field (bits 49-51) left at zero: the MMA takes
// the swizzle phase from the address bits themselves, as TMA does when it
// writes the tile (measured on B200: setting the field to the start's phase
// gives wrong products).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;             // leading byte offset (16 B units)
  d |= (uint64_t)(1024u >> 4) << 32;   // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1u << 46;             // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;             // SWIZZLE_128B
  return d;
}

// instruction descriptor (idesc_tr below): D f32 (bits 4-5), A/B format
// (bits 7-9 / 10-12: 0 f16, 1 bf16), K-major A and B, N >> 3 at bit 17,
// M >> 4 at bit 24

// byte offset of 16-byte chunk `chunk` of row `row` in a 128B-swizzled
// [rows x 128 B] tile (TMA SWIZZLE_128B pattern)
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)row * 128u + (uint32_t)((chunk ^ (row & 7)) << 4);
}

// ---------------------------------------------------------------------------
// 16-bit operand types: bf16 (the reference's compute dtype) or fp16
// ---------------------------------------------------------------------------

template <typename T>
struct F16Traits;
template <>
struct F16Traits<__nv_bfloat16> {
  static constexpr uint32_t kFormat = 1;  // tcgen05 kind::f16 operand format BF16
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&p);
  }
};
template <>
struct F16Traits<__half> {
  static constexpr uint32_t kFormat = 0;  // F16
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 p = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&p);
  }
};

// the transposed product of every layer: M = 128 output channels (A = a
// weight tile), N = 256 rows of a tile pair (B = the window)
template <typename T>
__host__ __device__ constexpr uint32_t idesc_tr() {
  return (1u << 4) | (F16Traits<T>::kFormat << 7) | (F16Traits<T>::kFormat << 10) | ((256u >> 3) << 17) |
         ((128u >> 4) << 24);
}

// ---------------------------------------------------------------------------
// convolution kernel
// ---------------------------------------------------------------------------

enum EpiMode : int { kEpiConv1 = 0, kEpiConv2 = 1, kEpiHeads = 2 };

// The fp32 residual stream x32 keeps each row's channels permuted within
// their 32-channel block: channel 32 q + 8 m + l (l < 8, m < 4) is stored
// at 32 q + 4 l + m.  An epilogue thread holds channels 32 q + l + 8 m for
// m < 4 (the mma fragment layout), so its four values of a row are one
// 16-byte vector.
__host__ __device__ constexpr int x32_slot(int c) { return (c & ~31) | ((c & 7) << 2) | ((c >> 3) & 3); }

struct EpiParams {
  int mode;
  int rows_valid;            // E * 100; rows at or above are padding
  int terms;                 // products per K step: 1; split operands 2 (A hi, lo) or 3 (+ W lo x A hi)
  const float *bias;         // [128] (BatchNorm after conv1 folded in)
  const float *bn_scale;     // conv2: next block's BN1 (or the final BN), per channel
  const float *bn_shift;
  const void *residual;      // conv2 / heads: x of the block input, [rows, 128] 16-bit
  float *x32;                // split operands: the fp32 residual stream [rows, 128] (channels in x32_slot order), updated in place
  int x32_natural_in;        // x32 is read in the natural channel order (the stem's output) and written in x32_slot order
  const float *head_w;       // heads: [6][128] 1x1 conv weights (head BN folded)
  const float *head_b;       // [6]
  float *head_out;           // heads: [rows, 8] f32
};

// Shared memory of conv_tc_kernel.  A tile pair is 256 output rows (two
// 128-row accumulators sharing every weight tile).  Its A operand for all
// nine taps is one window of 288 input rows (16 above the pair, 16 below;
// taps shift by at most 11) per 64-channel half, loaded once; a tap's A
// matrix is the window read from row 16 + 128 * sub + shift.  Weights
// stream through a ring of 16 KB (tap, half) tiles.
struct SmemLayout {
  static constexpr int kWinOff = 0;                                    // 2 halves x 36 KB
  static constexpr int kBOff = kWinOff + 2 * kWinHalfBytes;
  // staging tiles right after the weight ring, second output first: a
  // mode that leaves staging unused extends the ring into it (conv1 has one
  // output, 6 stages; the heads have none, 8 stages)
  static constexpr int kOut1Off = kBOff + kBStages * kBTileBytes;      // 2 halves x 16 KB
  static constexpr int kOut0Off = kOut1Off + 2 * kTileBytes;           // 2 halves x 16 KB
  static constexpr int kParamOff = kOut0Off + 2 * kTileBytes;          // floats
  static constexpr int kParamFloats = 3 * kC + kHeadCh * kC + 8;
  static constexpr int kHeadPartOff = kParamOff + kParamFloats * 4;  // [4 quads][128 rows][kHeadCh] floats
  static constexpr int kBarOff = kHeadPartOff + 4 * kBM * kHeadCh * 4;
  static constexpr int kNumBars = 2 + 2 + 2 * kMaxBStages + 2 + 2;
  static constexpr int kBytes = kBarOff + 8 * kNumBars + 16 + 1024;  // + alignment slack
};
static_assert(SmemLayout::kBOff % 1024 == 0 && SmemLayout::kOut1Off % 1024 == 0, "swizzled tiles 1024-aligned");
static_assert(kBTileBytes == kTileBytes, "weight stages and staging halves share a size");
static_assert(SmemLayout::kBytes <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ bool row_real(const EpiParams &ep, int r) {
  const int p = r % kRowsPerBoard;
  return r < ep.rows_valid && p >= 10 && (p % 10) != 9;
}

// The warp's 64 rows x 32 channels of the residual (conv2), global -> registers,
// issued before the staging buffer frees so their latency overlaps the wait.
template <typename T>
__device__ __forceinline__ void load_residual_tr(const EpiParams &ep, int tile, int quad, int wh, int lane,
                                                 uint4 (&res)[8]) {
  const T *base = static_cast<const T *>(ep.residual) + ((size_t)tile * kBM + wh * 64) * kC + quad * 32;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int idx = k * 32 + lane;
    res[k] = *reinterpret_cast<const uint4 *>(base + (size_t)(idx >> 2) * kC + (idx & 3) * 8);
  }
}

// One 128-row tile of a transposed accumulator (TMEM lane = output channel,
// column = row): bias / folded BatchNorm / ReLU / residual / next block's
// BN-ReLU exactly as epilogue_tile, computed in the fragment layout of
// tcgen05.ld 16x256b and written row-major into the 128B-swizzled staging
// tile by stmatrix .trans.  The warp covers channels 32 * quad + [0, 32)
// (its TMEM lane quadrant) and rows 64 * wh + [0, 64).  For conv2 the
// residual is first stored into out0 where its sum will go and read back
// in the fragment layout by ldmatrix .trans.  `cst` holds this thread's
// bias, BN scale and BN shift of channels 32 * quad + 8 m + lane / 4.
template <typename T>
__device__ __forceinline__ void epilogue_tile_tr(const EpiParams &ep, const float (&cst)[3][4], uint32_t acc_addr,
                                                 int tile, int quad, int wh, int lane, uint8_t *out0, uint8_t *out1,
                                                 const uint4 (&res)[8]) {
  const bool conv2 = ep.mode == kEpiConv2;
  uint8_t *h0 = out0 + (quad >> 1) * kTileBytes;
  uint8_t *h1 = out1 + (quad >> 1) * kTileBytes;
  const int row_base = wh * 64, chunk0 = (quad & 1) * 4;
  if (conv2) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int idx = k * 32 + lane;
      *reinterpret_cast<uint4 *>(h0 + swz(row_base + (idx >> 2), chunk0 + (idx & 3))) = res[k];
    }
    __syncwarp();
  }
  const int mrow = lane & 7, mat = lane >> 3;
  const uint32_t lane_addr = acc_addr + ((uint32_t)(quad * 32) << 16) + (uint32_t)row_base;
#pragma unroll 1
  for (int jj = 0; jj < 4; ++jj) {
    uint32_t d[2][2][4];  // [block of the two][lane group][fragment register]
#pragma unroll
    for (int j2 = 0; j2 < 2; ++j2)
#pragma unroll
      for (int g = 0; g < 2; ++g) tmem_ld16x256(lane_addr + ((uint32_t)(16 * g) << 16) + 8 * (2 * jj + j2), d[j2][g]);
    tmem_wait_ld();
#pragma unroll
    for (int j2 = 0; j2 < 2; ++j2) {
      const int rb = row_base + 8 * (2 * jj + j2);  // first row of the 8-row block in the tile
      const int r0 = tile * kBM + rb + 2 * (lane & 3);
      const bool real0 = row_real(ep, r0), real1 = row_real(ep, r0 + 1);
      const int srow = rb + mrow, schunk = chunk0 + mat;
      const uint32_t a0 = smem_u32(h0 + swz(srow, schunk));
      uint32_t rv[4] = {0u, 0u, 0u, 0u};
      if (conv2) ldmatrix_x4_trans(a0, rv);
      uint32_t p0[4], p1[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int g = m >> 1, hi = m & 1;
        const float y0 = __uint_as_float(d[j2][g][2 * hi]) + cst[0][m];
        const float y1 = __uint_as_float(d[j2][g][2 * hi + 1]) + cst[0][m];
        if (!conv2) {
          p0[m] = F16Traits<T>::pack(real0 ? fmaxf(y0, 0.0f) : 0.0f, real1 ? fmaxf(y1, 0.0f) : 0.0f);
        } else {
          const T *rh = reinterpret_cast<const T *>(&rv[m]);
          const float x0 = F16Traits<T>::to_f(F16Traits<T>::from_f(y0 + F16Traits<T>::to_f(rh[0])));
          const float x1 = F16Traits<T>::to_f(F16Traits<T>::from_f(y1 + F16Traits<T>::to_f(rh[1])));
          const float b0 = fmaxf(fmaf(x0, cst[1][m], cst[2][m]), 0.0f);
          const float b1 = fmaxf(fmaf(x1, cst[1][m], cst[2][m]), 0.0f);
          p0[m] = F16Traits<T>::pack(real0 ? x0 : 0.0f, real1 ? x1 : 0.0f);
          p1[m] = F16Traits<T>::pack(real0 ? b0 : 0.0f, real1 ? b1 : 0.0f);
        }
      }
      stmatrix_x4_trans(a0, p0);
      if (conv2) stmatrix_x4_trans(smem_u32(h1 + swz(srow, schunk)), p1);
    }
  }
}

// Split operands (terms >= 2): as epilogue_tile_tr, but every 16-bit output
// is written as a pair, hi = the value rounded to T into out0 and lo = the
// remainder (exact in fp32) rounded to T into out1, so hi + lo carries about
// twice T's significand into the next convolution; and the residual stream
// x stays fp32 in ep.x32 ([rows, 128] with each row's channels in x32_slot
// order, read and rewritten in place: a thread's four channels of a row are
// one 16-byte vector).  conv1 writes h's pair; conv2 writes
// x' = conv + bias + x to x32 and the pair of relu(bn(x')).
template <typename T>
__device__ __forceinline__ void epilogue_tile_tr_split(const EpiParams &ep, const float (&cst)[3][4],
                                                       uint32_t acc_addr, int tile, int quad, int wh, int lane,
                                                       uint8_t *out0, uint8_t *out1) {
  const bool conv2 = ep.mode == kEpiConv2;
  uint8_t *h0 = out0 + (quad >> 1) * kTileBytes;
  uint8_t *h1 = out1 + (quad >> 1) * kTileBytes;
  const int row_base = wh * 64, chunk0 = (quad & 1) * 4;
  const int mrow = lane & 7, mat = lane >> 3;
  const uint32_t lane_addr = acc_addr + ((uint32_t)(quad * 32) << 16) + (uint32_t)row_base;
  const int ch0 = quad * 32 + lane / 4;  // + 8 m: this thread's channels
  const int xs = x32_slot(ch0);          // their four x32 slots, xs .. xs + 3
  // Software pipeline over the four 16-row steps jj: the accumulator
  // columns and the residual of step jj + 1 are requested before step jj
  // is computed, so their latency hides behind that step's arithmetic
  // (tcgen05.wait::ld then only waits for loads issued a step earlier).
  uint32_t d[2][2][2][4];  // [buffer][block of the two][lane group][fragment register]
  float rx[2][2][4][2];    // [buffer][block][m][row of the pair]
  auto request = [&](int jj, int buf) {
#pragma unroll
    for (int j2 = 0; j2 < 2; ++j2)
#pragma unroll
      for (int g = 0; g < 2; ++g)
        tmem_ld16x256(lane_addr + ((uint32_t)(16 * g) << 16) + 8 * (2 * jj + j2), d[buf][j2][g]);
    if (conv2) {
#pragma unroll
      for (int j2 = 0; j2 < 2; ++j2) {
        const size_t r0 = (size_t)tile * kBM + row_base + 8 * (2 * jj + j2) + 2 * (lane & 3);
        if (ep.x32_natural_in) {
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            rx[buf][j2][m][0] = ep.x32[r0 * kC + ch0 + 8 * m];
            rx[buf][j2][m][1] = ep.x32[(r0 + 1) * kC + ch0 + 8 * m];
          }
        } else {
          const float4 v0 = *reinterpret_cast<const float4 *>(ep.x32 + r0 * kC + xs);
          const float4 v1 = *reinterpret_cast<const float4 *>(ep.x32 + (r0 + 1) * kC + xs);
          rx[buf][j2][0][0] = v0.x;
          rx[buf][j2][1][0] = v0.y;
          rx[buf][j2][2][0] = v0.z;
          rx[buf][j2][3][0] = v0.w;
          rx[buf][j2][0][1] = v1.x;
          rx[buf][j2][1][1] = v1.y;
          rx[buf][j2][2][1] = v1.z;
          rx[buf][j2][3][1] = v1.w;
        }
      }
    }
  };
  request(0, 0);
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    const int cur = jj & 1;
    tmem_wait_ld();
    if (jj + 1 < 4) request(jj + 1, cur ^ 1);
#pragma unroll
    for (int j2 = 0; j2 < 2; ++j2) {
      const int rb = row_base + 8 * (2 * jj + j2);  // first row of the 8-row block in the tile
      const int r0 = tile * kBM + rb + 2 * (lane & 3);
      const bool real0 = row_real(ep, r0), real1 = row_real(ep, r0 + 1);
      const int srow = rb + mrow, schunk = chunk0 + mat;
      uint32_t p0[4], p1[4];
      float xn[2][4];  // conv2: the updated residual of rows r0, r0 + 1
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int g = m >> 1, hi = m & 1;
        const float y0 = __uint_as_float(d[cur][j2][g][2 * hi]) + cst[0][m];
        const float y1 = __uint_as_float(d[cur][j2][g][2 * hi + 1]) + cst[0][m];
        float v0, v1;
        if (!conv2) {
          v0 = real0 ? fmaxf(y0, 0.0f) : 0.0f;
          v1 = real1 ? fmaxf(y1, 0.0f) : 0.0f;
        } else {
          const float x0 = real0 ? y0 + rx[cur][j2][m][0] : 0.0f;
          const float x1 = real1 ? y1 + rx[cur][j2][m][1] : 0.0f;
          xn[0][m] = x0;
          xn[1][m] = x1;
          v0 = real0 ? fmaxf(fmaf(x0, cst[1][m], cst[2][m]), 0.0f) : 0.0f;
          v1 = real1 ? fmaxf(fmaf(x1, cst[1][m], cst[2][m]), 0.0f) : 0.0f;
        }
        const float a0 = F16Traits<T>::to_f(F16Traits<T>::from_f(v0));
        const float a1 = F16Traits<T>::to_f(F16Traits<T>::from_f(v1));
        p0[m] = F16Traits<T>::pack(a0, a1);
        p1[m] = F16Traits<T>::pack(v0 - a0, v1 - a1);
      }
      if (conv2) {
        *reinterpret_cast<float4 *>(ep.x32 + (size_t)r0 * kC + xs) =
            make_float4(xn[0][0], xn[0][1], xn[0][2], xn[0][3]);
        *reinterpret_cast<float4 *>(ep.x32 + (size_t)(r0 + 1) * kC + xs) =
            make_float4(xn[1][0], xn[1][1], xn[1][2], xn[1][3]);
      }
      stmatrix_x4_trans(smem_u32(h0 + swz(srow, schunk)), p0);
      stmatrix_x4_trans(smem_u32(h1 + swz(srow, schunk)), p1);
    }
  }
}

// The head layer (the last block's conv2) in the transposed layout: the
// residual sum and the trunk's final BN + ReLU as in conv2, then the six 1x1
// head channels per row.  Each thread sums its 4 channels' products for its
// two rows of every 8-row block, the 8 lanes of a row pair add theirs with
// an xor butterfly, and lanes 0-3 leave the warp's 32-channel partials in
// `part` [quad][row][head]; store_heads_tr then adds the four quads in
// order.  Without split operands the residual is 16-bit and staged through
// out0 (as conv2); with them it is the fp32 stream, read element by element,
// and the heads read the fp32 activation.
template <typename T, bool Split>
__device__ __forceinline__ void epilogue_tile_tr_heads(const EpiParams &ep, const float (&cst)[3][4],
                                                       const float *prm, uint32_t acc_addr, int tile, int quad,
                                                       int wh, int lane, uint8_t *out0, const uint4 (&res)[8],
                                                       float *part) {
  uint8_t *h0 = out0 + (quad >> 1) * kTileBytes;
  const int row_base = wh * 64, chunk0 = (quad & 1) * 4;
  if (!Split) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int idx = k * 32 + lane;
      *reinterpret_cast<uint4 *>(h0 + swz(row_base + (idx >> 2), chunk0 + (idx & 3))) = res[k];
    }
    __syncwarp();
  }
  const int mrow = lane & 7, mat = lane >> 3;
  const uint32_t lane_addr = acc_addr + ((uint32_t)(quad * 32) << 16) + (uint32_t)row_base;
  const int ch0 = quad * 32 + lane / 4;  // + 8 m: this thread's channels
  float hw[kHeadCh][4];
#pragma unroll
  for (int h = 0; h < kHeadCh; ++h)
#pragma unroll
    for (int m = 0; m < 4; ++m) hw[h][m] = prm[3 * kC + h * kC + ch0 + 8 * m];
#pragma unroll 1
  for (int jj = 0; jj < 4; ++jj) {
    uint32_t d[2][2][4];
#pragma unroll
    for (int j2 = 0; j2 < 2; ++j2)
#pragma unroll
      for (int g = 0; g < 2; ++g) tmem_ld16x256(lane_addr + ((uint32_t)(16 * g) << 16) + 8 * (2 * jj + j2), d[j2][g]);
    float rx[2][4][2];
    if (Split) {
#pragma unroll
      for (int j2 = 0; j2 < 2; ++j2) {
        const size_t r0 = (size_t)tile * kBM + row_base + 8 * (2 * jj + j2) + 2 * (lane & 3);
        if (ep.x32_natural_in) {
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            rx[j2][m][0] = ep.x32[r0 * kC + ch0 + 8 * m];
            rx[j2][m][1] = ep.x32[(r0 + 1) * kC + ch0 + 8 * m];
          }
        } else {
          const float4 v0 = *reinterpret_cast<const float4 *>(ep.x32 + r0 * kC + x32_slot(ch0));
          const float4 v1 = *reinterpret_cast<const float4 *>(ep.x32 + (r0 + 1) * kC + x32_slot(ch0));
          rx[j2][0][0] = v0.x;
          rx[j2][1][0] = v0.y;
          rx[j2][2][0] = v0.z;
          rx[j2][3][0] = v0.w;
          rx[j2][0][1] = v1.x;
          rx[j2][1][1] = v1.y;
          rx[j2][2][1] = v1.z;
          rx[j2][3][1] = v1.w;
        }
      }
    }
    tmem_wait_ld();
#pragma unroll
    for (int j2 = 0; j2 < 2; ++j2) {
      const int rb = row_base + 8 * (2 * jj + j2);
      const int r0 = tile * kBM + rb + 2 * (lane & 3);
      const bool real0 = row_real(ep, r0), real1 = row_real(ep, r0 + 1);
      if (!Split) {
        uint32_t rv[4];
        ldmatrix_x4_trans(smem_u32(h0 + swz(rb + mrow, chunk0 + mat)), rv);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const T *rh = reinterpret_cast<const T *>(&rv[m]);
          rx[j2][m][0] = F16Traits<T>::to_f(rh[0]);
          rx[j2][m][1] = F16Traits<T>::to_f(rh[1]);
        }
      }
      float acc[kHeadCh][2];
#pragma unroll
      for (int h = 0; h < kHeadCh; ++h) acc[h][0] = acc[h][1] = 0.0f;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int g = m >> 1, hi = m & 1;
        const float y0 = __uint_as_float(d[j2][g][2 * hi]) + cst[0][m];
        const float y1 = __uint_as_float(d[j2][g][2 * hi + 1]) + cst[0][m];
        float x0 = y0 + rx[j2][m][0], x1 = y1 + rx[j2][m][1];
        if (!Split) {
          // residual stream in the 16-bit type, heads on the 16-bit activation
          x0 = F16Traits<T>::to_f(F16Traits<T>::from_f(x0));
          x1 = F16Traits<T>::to_f(F16Traits<T>::from_f(x1));
        }
        float a0 = real0 ? fmaxf(fmaf(x0, cst[1][m], cst[2][m]), 0.0f) : 0.0f;
        float a1 = real1 ? fmaxf(fmaf(x1, cst[1][m], cst[2][m]), 0.0f) : 0.0f;
        if (!Split) {
          a0 = F16Traits<T>::to_f(F16Traits<T>::from_f(a0));
          a1 = F16Traits<T>::to_f(F16Traits<T>::from_f(a1));
        }
#pragma unroll
        for (int h = 0; h < kHeadCh; ++h) {
          acc[h][0] = fmaf(a0, hw[h][m], acc[h][0]);
          acc[h][1] = fmaf(a1, hw[h][m], acc[h][1]);
        }
      }
      // add the 8 lanes of this row pair (lane / 4 = channel within 8) by
      // reduce-scatter: 16 slots (head h, row i at 2 h + i; 12-15 empty),
      // each xor step keeps the half named by this lane's bit and adds the
      // partner's copy of it, so lane q = lane / 4 ends with head q's two rows
      float v[16];
#pragma unroll
      for (int h = 0; h < kHeadCh; ++h) {
        v[2 * h] = acc[h][0];
        v[2 * h + 1] = acc[h][1];
      }
#pragma unroll
      for (int k = 2 * kHeadCh; k < 16; ++k) v[k] = 0.0f;
#pragma unroll
      for (int step = 0, width = 8; step < 3; ++step, width >>= 1) {
        const int off = 16 >> step;          // lane bits 4, 3, 2
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (k < width) {
            const float send = upper ? v[k] : v[width + k];
            const float keep = upper ? v[width + k] : v[k];
            v[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
          }
        }
      }
      const int q = lane >> 2;
      if (q < kHeadCh) {
        const int row = rb + 2 * (lane & 3);
        part[(quad * kBM + row) * kHeadCh + q] = v[0];
        part[(quad * kBM + row + 1) * kHeadCh + q] = v[1];
      }
    }
  }
}

// heads: a row's four quad partials in order, bias, ReLU
__device__ __forceinline__ void store_heads_tr(const EpiParams &ep, const float *prm, int tile, int row_in_tile,
                                               const float *part) {
  const int r = tile * kBM + row_in_tile;
  if (r >= ep.rows_valid) return;
  const bool real = row_real(ep, r);
  float hb[kHeadCh];
#pragma unroll
  for (int h = 0; h < kHeadCh; ++h) {
    float v = part[(0 * kBM + row_in_tile) * kHeadCh + h];
#pragma unroll
    for (int q = 1; q < 4; ++q) v += part[(q * kBM + row_in_tile) * kHeadCh + h];
    hb[h] = real ? fmaxf(v + prm[3 * kC + kHeadCh * kC + h], 0.0f) : 0.0f;
  }
  float4 *dst = reinterpret_cast<float4 *>(ep.head_out + (size_t)r * 8);
  dst[0] = make_float4(hb[0], hb[1], hb[2], hb[3]);
  dst[1] = make_float4(hb[4], hb[5], 0.0f, 0.0f);
}

// Split operands (Split, ep.terms 2 or 3): the activation comes as two
// 16-bit matrices, hi and lo, and a pair's K loop runs over four windows
// (hi and lo of each 64-channel half) through the same two window slots.
// Per (window, tap) the weight tiles are W_hi, plus W_lo after W_hi for a
// hi window when terms = 3, so the accumulator receives W_hi A_hi +
// W_hi A_lo (+ W_lo A_hi): the product of the split operands up to the
// lo x lo term.  The weight map then holds [terms == 3 ? 2 : 1][9 taps]
// [128 out][128 in].
template <typename T, bool Split>
__global__ void __launch_bounds__(kThreads, 1) conv_tc_kernel(const __grid_constant__ CUtensorMap tm_win,
                                                              const __grid_constant__ CUtensorMap tm_win_lo,
                                                              const __grid_constant__ CUtensorMap tm_w,
                                                              const __grid_constant__ CUtensorMap tm_out0,
                                                              const __grid_constant__ CUtensorMap tm_out1,
                                                              EpiParams ep, int num_tiles) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int num_pairs = (num_tiles + 1) / 2;
  float *prm = reinterpret_cast<float *>(smem + SmemLayout::kParamOff);
  uint64_t *win_full = reinterpret_cast<uint64_t *>(smem + SmemLayout::kBarOff);
  uint64_t *win_empty = win_full + 2;
  uint64_t *b_full = win_empty + 2;
  uint64_t *b_empty = b_full + kMaxBStages;
  uint64_t *acc_full = b_empty + kMaxBStages;
  // weight stages: the staging tiles an epilogue mode leaves unused extend the ring
  // (the head layer stages a 16-bit residual through out0; split operands
  // read theirs from the fp32 stream and leave both staging tiles unused)
  const int nbs = ep.mode == kEpiHeads ? (Split ? kMaxBStages : kBStages + 2)
                                       : (ep.mode == kEpiConv1 && !Split ? 6 : kBStages);
  // windows per pair (hi and lo of each half with split operands) and the
  // weight tiles per (window, tap)
  const int nwin = Split ? 4 : 2;
  const int wlo_terms = Split && ep.terms == 3 ? 2 : 1;  // weight tiles per tap of a hi window
  uint64_t *acc_empty = acc_full + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  // epilogue constants into shared memory
  for (int i = threadIdx.x; i < kC; i += kThreads) {
    prm[i] = ep.bias[i];
    prm[kC + i] = ep.bn_scale ? ep.bn_scale[i] : 1.0f;
    prm[2 * kC + i] = ep.bn_shift ? ep.bn_shift[i] : 0.0f;
  }
  if (ep.mode == kEpiHeads) {
    for (int i = threadIdx.x; i < kHeadCh * kC; i += kThreads) prm[3 * kC + i] = ep.head_w[i];
    if (threadIdx.x < kHeadCh) prm[3 * kC + kHeadCh * kC + threadIdx.x] = ep.head_b[threadIdx.x];
  }
  if (threadIdx.x == 0) {
    for (int h = 0; h < 2; ++h) {
      mbar_init(&win_full[h], 1);
      mbar_init(&win_empty[h], 1);
    }
    for (int s = 0; s < kMaxBStages; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kEpiThreads);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- weight producer ----------------
    if (lane == 0) {
      int bstage = 0;
      uint32_t bphase = 0, b_issued = 0, b_parity = 0;  // per stage: issued?, parity of the last load
      bool stop = false;
      for (int pair = blockIdx.x; pair < num_pairs && !stop && !*abort_flag; pair += gridDim.x) {
        for (int wi = 0; wi < nwin && !stop; ++wi) {
          const int h = Split ? wi >> 1 : wi;
          const int nt = Split && (wi & 1) ? 1 : wlo_terms;
          for (int tap = 0; tap < 9 && !stop; ++tap) {
            for (int term = 0; term < nt; ++term) {
              if (!mbar_wait(&b_empty[bstage], bphase ^ 1u, abort_flag)) {
                stop = true;
                break;
              }
              uint8_t *sb = smem + SmemLayout::kBOff + bstage * kBTileBytes;
              mbar_expect_tx(&b_full[bstage], kBTileBytes);
              tma_load_2d(sb, &tm_w, &b_full[bstage], h * kBK, (term * 9 + tap) * kC);
              b_issued |= 1u << bstage;
              b_parity = (b_parity & ~(1u << bstage)) | (bphase << bstage);
              if (++bstage == nbs) {
                bstage = 0;
                bphase ^= 1u;
              }
            }
          }
        }
      }
      // every load issued into shared memory lands before the CTA may exit
      for (int s = 0; s < nbs; ++s)
        if (b_issued >> s & 1u) mbar_drain(&b_full[s], b_parity >> s & 1u);
    }
  } else if (warp == kThreads / 32 - 1) {
    // ---------------- window producer ----------------
    // Its own warp, so a window half reloads as soon as the MMAs release it
    // (a whole half of the pair ahead) instead of queueing behind weights.
    if (lane == 0) {
      uint32_t wphase[2] = {0u, 0u}, w_issued = 0, w_parity = 0;
      bool stop = false;
      for (int pair = blockIdx.x; pair < num_pairs && !stop && !*abort_flag; pair += gridDim.x) {
        const int row0 = pair * 2 * kBM;
        for (int wi = 0; wi < nwin; ++wi) {
          const int s = wi & 1;                      // window slot
          const int h = Split ? wi >> 1 : wi;        // channel half
          const CUtensorMap *src = Split && (wi & 1) ? &tm_win_lo : &tm_win;
          if (!mbar_wait(&win_empty[s], wphase[s] ^ 1u, abort_flag)) {
            stop = true;
            break;
          }
          uint8_t *win = smem + SmemLayout::kWinOff + s * kWinHalfBytes;
          mbar_expect_tx(&win_full[s], kWinHalfBytes);
          tma_load_2d(win, src, &win_full[s], h * kBK, row0 - kWinLead);
          tma_load_2d(win + kWinBoxRows * 128, src, &win_full[s], h * kBK, row0 - kWinLead + kWinBoxRows);
          w_issued |= 1u << s;
          w_parity = (w_parity & ~(1u << s)) | (wphase[s] << s);
          wphase[s] ^= 1u;
        }
      }
      for (int h = 0; h < 2; ++h)
        if (w_issued >> h & 1u) mbar_drain(&win_full[h], w_parity >> h & 1u);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int bstage = 0, slot = 0;
      uint32_t bphase = 0, acc_phase = 0, wphase[2] = {0u, 0u};
      for (int pair = blockIdx.x; pair < num_pairs && !*abort_flag; pair += gridDim.x) {
        if (!mbar_wait(&acc_empty[slot], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d0 = tmem_base + (uint32_t)(2 * slot * kC);
        bool ok = true;
        for (int wi = 0; wi < nwin && ok; ++wi) {
          const int s = wi & 1;
          const int nt = Split && (wi & 1) ? 1 : wlo_terms;
          if (!mbar_wait(&win_full[s], wphase[s], abort_flag)) {
            ok = false;
            break;
          }
          wphase[s] ^= 1u;
          tc_fence_after();
          const uint32_t win = smem_u32(smem + SmemLayout::kWinOff + s * kWinHalfBytes);
          for (int tap = 0; tap < 9 && ok; ++tap) {
            const int off = (tap / 3 - 1) * 10 + (tap % 3 - 1);
            for (int term = 0; term < nt; ++term) {
              if (!mbar_wait(&b_full[bstage], bphase, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t sb = smem_u32(smem + SmemLayout::kBOff + bstage * kBTileBytes);
              const uint32_t acc = (wi | tap | term) != 0;
              // D[channel][row] of both sub-tiles: one N = 256 product per K step
              const uint32_t wrow = win + (uint32_t)(kWinLead + off) * 128u;
#pragma unroll
              for (int k = 0; k < kBK / 16; ++k)
                umma_f16(d0, smem_desc_sw128(sb + k * 32), smem_desc_sw128(wrow + k * 32), idesc_tr<T>(),
                         acc | (k != 0));
              umma_commit(&b_empty[bstage]);
              if (++bstage == nbs) {
                bstage = 0;
                bphase ^= 1u;
              }
            }
          }
          if (ok) umma_commit(&win_empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[slot]);
        if (++slot == 2) {
          slot = 0;
          acc_phase ^= 1u;
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2-9) ----------------
    const int quad = warp & 3;              // TMEM lanes this warp may access
    const int half = (warp - 2) >> 2;       // column half: warps 2-5 -> 0, 6-9 -> 1
    const int et = threadIdx.x - 64;        // 0..255
    uint8_t *out0 = smem + SmemLayout::kOut0Off;
    uint8_t *out1 = smem + SmemLayout::kOut1Off;
    float *head_part = reinterpret_cast<float *>(smem + SmemLayout::kHeadPartOff);
    volatile int *go = abort_flag + 1;  // elected thread's verdict for the pair
    int slot = 0;
    uint32_t acc_phase = 0;
    float cst[3][4];  // transposed epilogue: bias, BN scale, BN shift of this thread's channels
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int ch = quad * 32 + 8 * m + lane / 4;
      cst[0][m] = prm[ch];
      cst[1][m] = prm[kC + ch];
      cst[2][m] = prm[2 * kC + ch];
    }
    // the residual of a pair is read by the epilogue only: prefetch it into
    // L2 when this CTA's previous pair is done, so its loads do not wait on
    // HBM.  That is about one mainloop ahead; a whole pair period ahead,
    // the streaming traffic evicted a third of the prefetched lines before
    // the epilogue read them (conv2 read 1.20 GB per 8192-board launch
    // instead of 0.86).
    const bool has_res = ep.mode != kEpiConv1;
    auto prefetch_residual = [&](int p) {
      for (int sub = 0; sub < 2; ++sub) {
        const int tile = p * 2 + sub;
        if (p < num_pairs && tile < num_tiles) {
          if (Split)
            prefetch_l2(ep.x32 + (size_t)tile * kBM * kC, kBM * kC * (uint32_t)sizeof(float));
          else
            prefetch_l2(static_cast<const T *>(ep.residual) + (size_t)tile * kBM * kC,
                        kBM * kC * (uint32_t)sizeof(T));
        }
      }
    };
    if (has_res && et == 0) prefetch_residual(blockIdx.x);
    for (int pair = blockIdx.x; pair < num_pairs; pair += gridDim.x) {
      // one thread waits (bounded) and broadcasts, so the epilogue threads agree
      if (et == 0) {
        const bool ok = !*abort_flag && mbar_wait(&acc_full[slot], acc_phase, abort_flag);
        *go = ok ? 1 : 0;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      if (!*go) break;
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");  // everyone read `go` before it changes
      tc_fence_after();
      for (int sub = 0; sub < 2; ++sub) {
        const int tile = pair * 2 + sub;
        if (tile >= num_tiles) break;  // uniform across the epilogue threads
        uint4 res[8];
        if (!Split && ep.mode != kEpiConv1) load_residual_tr<T>(ep, tile, quad, half, lane, res);
        if (ep.mode != kEpiHeads) {
          // the staging buffers are free once the previous store has read them
          if (et == 0) tma_store_wait_read();
          asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
        }
        const uint32_t acc_addr = tmem_base + (uint32_t)((2 * slot + sub) * kC);
        if (ep.mode == kEpiHeads) {
          epilogue_tile_tr_heads<T, Split>(ep, cst, prm, acc_addr, tile, quad, half, lane, out0, res, head_part);
          asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
          if (et < kBM) store_heads_tr(ep, prm, tile, et, head_part);
          asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");  // partials and staging consumed
          continue;
        }
        if (Split)
          epilogue_tile_tr_split<T>(ep, cst, acc_addr, tile, quad, half, lane, out0, out1);
        else
          epilogue_tile_tr<T>(ep, cst, acc_addr, tile, quad, half, lane, out0, out1, res);
        fence_proxy_async();
        asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
        if (et == 0) {
          const int row0 = tile * kBM;
          tma_store_2d(&tm_out0, out0, 0, row0);
          tma_store_2d(&tm_out0, out0 + kTileBytes, kBK, row0);
          if (ep.mode == kEpiConv2 || Split) {
            tma_store_2d(&tm_out1, out1, 0, row0);
            tma_store_2d(&tm_out1, out1 + kTileBytes, kBK, row0);
          }
          tma_store_commit();
        }
      }
      // both accumulators of the pair can be reused by the MMA warp
      tc_fence_before();
      mbar_arrive(&acc_empty[slot]);
      if (has_res && et == 0) prefetch_residual(pair + gridDim.x);
      if (++slot == 2) {
        slot = 0;
        acc_phase ^= 1u;
      }
    }
    if (et == 0) tma_store_wait_all();
  }
  // every role has left its loop (all waits are bounded) and the producer
  // has drained its loads; the MMA warp's last commits landed on barriers
  // the epilogue waited for (or the kernel is aborting)
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// stem: conv3x3 in_planes -> 128 (+ bias), then BN1 of block 0 and ReLU.
// A CTA serves kStemBoards boards; each thread computes 8 adjacent
// channels of one row (16 threads cover a row, so a warp stores two full
// 256-byte rows per output).  For observations of {0, 1} planes (at most
// 4) a tap costs one row of a table of per-tap weight sums over the 16
// plane subsets, instead of a product per plane; the table is built once
// per forward by stem_table_kernel and read through the L1 cache.  Other
// inputs take the direct products.
// ---------------------------------------------------------------------------

constexpr int kStemBoards = 8;
constexpr int kStemThreads = 256;
constexpr int kStemSubsets = 16;  // plane subsets of up to 4 planes
constexpr size_t kStemTableBytes = (size_t)9 * kStemSubsets * kC * sizeof(float);

size_t stem_smem_bytes(int) { return (size_t)kStemBoards * 128; }

// The subset table [9 taps][16 subsets][128]: entry (tap, m) sums the
// weights of the planes in m in increasing plane order.  A table row keeps
// channel n = 8 g + 4 j + l at 64 j + 4 g + l, so the 16 threads of a stem
// row read 256 contiguous bytes per float4 load.
__global__ void __launch_bounds__(256) stem_table_kernel(int in_planes, const float *w, float *table) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 9 * kStemSubsets * kC; i += gridDim.x * blockDim.x) {
    const int k = i % kC, m = (i / kC) % kStemSubsets, tap = i / (kStemSubsets * kC);
    const int n = ((k & 63) >> 2) * 8 + (k >> 6) * 4 + (k & 3);
    float v = 0.0f;
    bool any = false;
    for (int c = 0; c < in_planes; ++c)
      if (m >> c & 1) {
        const float wv = w[(tap * in_planes + c) * kC + n];
        v = any ? v + wv : wv;
        any = true;
      }
    table[i] = v;  // subsets naming planes >= in_planes are never looked up
  }
}

// With split operands (Split) x is written in fp32 to x32 and a as the
// pair a (hi) / a_lo of 16-bit matrices.
template <typename T, bool Split>
__global__ void __launch_bounds__(kStemThreads, 3) stem_kernel(const float *obs, int boards, int in_planes,
                                                            const float *w, const float *sw, const float *b,
                                                            const float *s1, const float *t1, T *x, T *a,
                                                            float *x32, T *a_lo) {
  extern __shared__ float sm[];
  const bool table = in_planes <= 4;
  // sw: the subset table [9 taps][16 subsets][128] (table), else unused;
  // w: the weights [9 * in_planes][128]
  uint8_t *masks = reinterpret_cast<uint8_t *>(sm);  // [boards][11 * 11]
  const int e0 = blockIdx.x * kStemBoards;
  const int nb = min(kStemBoards, boards - e0);
  // plane-subset mask per cell on an 11 x 11 grid with a zero border
  int binary = table ? 1 : 0;
  if (table) {
    for (int i = threadIdx.x; i < nb * 121; i += kStemThreads) {
      const int eb = i / 121, q = i % 121, yy = q / 11 - 1, xx = q % 11 - 1;
      uint32_t m = 0;
      if (yy >= 0 && yy < 9 && xx >= 0 && xx < 9) {
        const float *o = obs + ((size_t)(e0 + eb) * 81 + yy * 9 + xx) * in_planes;
        for (int c = 0; c < in_planes; ++c) {
          const float v = o[c];
          if (v == 1.0f) m |= 1u << c;
          else if (v != 0.0f) binary = 0;
        }
      }
      masks[eb * 128 + q] = (uint8_t)m;
    }
  }
  binary = __syncthreads_and(binary);
  const int g = threadIdx.x & 15, n0 = g * 8;  // this thread's 8 channels
  float bias[8], sc[8], sh[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    bias[j] = b[n0 + j];
    sc[j] = s1[n0 + j];
    sh[j] = t1[n0 + j];
  }
  for (int item = threadIdx.x >> 4; item < kStemBoards * kRowsPerBoard; item += kStemThreads >> 4) {
    const int eb = item / kRowsPerBoard, p = item - eb * kRowsPerBoard;
    if (eb >= nb) break;
    const int yp = p / 10, xp = p - yp * 10;
    const bool real = yp >= 1 && xp <= 8;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = bias[j];
    if (real) {
      const int y = yp - 1, xx = xp;
      if (binary) {
        const uint8_t *mb = masks + eb * 128;
#pragma unroll
        for (int tap = 0; tap < 9; ++tap) {
          const int m = mb[(y + tap / 3) * 11 + (xx + tap % 3)];
          if (m == 0) continue;
          const float *lt = sw + (tap * kStemSubsets + m) * kC + 4 * g;
          const float4 l0 = __ldg(reinterpret_cast<const float4 *>(lt));
          const float4 l1 = __ldg(reinterpret_cast<const float4 *>(lt + 64));
          acc[0] += l0.x;
          acc[1] += l0.y;
          acc[2] += l0.z;
          acc[3] += l0.w;
          acc[4] += l1.x;
          acc[5] += l1.y;
          acc[6] += l1.z;
          acc[7] += l1.w;
        }
      } else {
        for (int ky = 0; ky < 3; ++ky) {
          const int iy = y + ky - 1;
          if (iy < 0 || iy >= 9) continue;
          for (int kx = 0; kx < 3; ++kx) {
            const int ix = xx + kx - 1;
            if (ix < 0 || ix >= 9) continue;
            const int tap = ky * 3 + kx;
            const float *o = obs + ((size_t)(e0 + eb) * 81 + iy * 9 + ix) * in_planes;
            for (int c = 0; c < in_planes; ++c) {
              const float ov = o[c];
              if (table) {
                const float *wt = sw + (tap * kStemSubsets + (1 << c)) * kC + 4 * g;
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[j] = fmaf(ov, __ldg(wt + (j >> 2) * 64 + (j & 3)), acc[j]);
              } else {
                const float *wt = w + (tap * in_planes + c) * kC + n0;
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[j] = fmaf(ov, __ldg(wt + j), acc[j]);
              }
            }
          }
        }
      }
    }
    const size_t r = (size_t)(e0 + eb) * kRowsPerBoard + p;
    if (Split) {
      // fp32 x; a as hi + lo
      float xv[8];
      uint32_t ph[4], pl[4];
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        float hi[2], lo[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          xv[j + u] = real ? acc[j + u] : 0.0f;
          const float av = real ? fmaxf(fmaf(xv[j + u], sc[j + u], sh[j + u]), 0.0f) : 0.0f;
          hi[u] = F16Traits<T>::to_f(F16Traits<T>::from_f(av));
          lo[u] = av - hi[u];
        }
        ph[j / 2] = F16Traits<T>::pack(hi[0], hi[1]);
        pl[j / 2] = F16Traits<T>::pack(lo[0], lo[1]);
      }
      // x32 in the natural channel order: the first block's conv2 reads it
      // so and writes the permuted order (x32_slot)
      float4 *xd = reinterpret_cast<float4 *>(x32 + r * kC + n0);
      xd[0] = make_float4(xv[0], xv[1], xv[2], xv[3]);
      xd[1] = make_float4(xv[4], xv[5], xv[6], xv[7]);
      *reinterpret_cast<uint4 *>(a + r * kC + n0) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
      *reinterpret_cast<uint4 *>(a_lo + r * kC + n0) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
    } else {
      uint32_t px[4], pa[4];
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        float xv[2], av[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const float xr = F16Traits<T>::to_f(F16Traits<T>::from_f(real ? acc[j + u] : 0.0f));
          xv[u] = xr;
          av[u] = real ? fmaxf(fmaf(xr, sc[j + u], sh[j + u]), 0.0f) : 0.0f;
        }
        px[j / 2] = F16Traits<T>::pack(xv[0], xv[1]);
        pa[j / 2] = F16Traits<T>::pack(av[0], av[1]);
      }
      *reinterpret_cast<uint4 *>(x + r * kC + n0) = make_uint4(px[0], px[1], px[2], px[3]);
      *reinterpret_cast<uint4 *>(a + r * kC + n0) = make_uint4(pa[0], pa[1], pa[2], pa[3]);
    }
  }
}

// ---------------------------------------------------------------------------
// heads: the linears on the 1x1-conv features, then dirichlet_from_logits
// (network.py:150-212, log-concentration heads).  A CTA serves
// kHeadBoards boards so every weight it reads feeds all of them; each
// dot product keeps one fixed summation order.
// ---------------------------------------------------------------------------

constexpr int kHeadBoards = 16;
constexpr int kHeadHalf = kHeadBoards / 2;  // boards per thread: two threads share an output
constexpr int kHeadThreads = 256;
constexpr int kFeat = 81 * kHeadCh;

struct HeadWeights {
  int A;
  const float *policy_w, *policy_b;          // [162][A], [A]
  const float *value_w1, *value_b1;          // [81][128], [128]
  const float *value_mean_w, *value_mean_b;  // [128][2], [2]
  const float *value_conc_w, *value_conc_b;  // [128], [1]
  const float *qdir_w1, *qdir_b1;            // [162][128], [128]
  const float *qdir_w2, *qdir_b2;            // [128][2A], [2A]
  const float *qconc_w1, *qconc_b1;          // [81][128], [128]
  const float *qconc_w2, *qconc_b2;          // [128][A], [A]
};

// the features' region, reused for the Q heads' outputs once the hidden
// layers have read the features
__host__ __device__ inline int head_shared_floats(int A) { return kFeat > 3 * A ? kFeat : 3 * A; }

size_t head_smem_bytes(int A) {
  return (size_t)kHeadBoards * (head_shared_floats(A) + 3 * kC) * sizeof(float);
}

// sum over k < 128 of h[k * hstride] * w[k * stride]: lanes 32-wide
// butterflies per 32-element block, blocks added in order
__device__ __forceinline__ float warp_dot128(const float *h, int hstride, const float *w, int stride, int lane) {
  float total = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float v = h[(j * 32 + lane) * hstride] * w[(j * 32 + lane) * stride];
    for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    total = j == 0 ? v : total + v;
  }
  return total;
}

// acc[g] += x[k][g] * wv for the G = 16 boards of x's row k (boards
// innermost, read as four broadcast float4s)
// acc[g] += xk[g] * wv for this thread's kHeadHalf boards (xk already
// offset to them): two float4 broadcasts per k
__device__ __forceinline__ void fma_boards(float (&acc)[kHeadHalf], const float *xk, float wv) {
  static_assert(kHeadHalf == 8, "two float4 per row");
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const float4 v = *reinterpret_cast<const float4 *>(xk + 4 * q);
    acc[4 * q] = fmaf(v.x, wv, acc[4 * q]);
    acc[4 * q + 1] = fmaf(v.y, wv, acc[4 * q + 1]);
    acc[4 * q + 2] = fmaf(v.z, wv, acc[4 * q + 2]);
    acc[4 * q + 3] = fmaf(v.w, wv, acc[4 * q + 3]);
  }
}

// Shared arrays keep the boards innermost ([k][G]), so one float4
// broadcast feeds four boards' products; each output's sum over k keeps
// its fixed order.  Two threads share an output, one per half of the
// CTA's boards (thread t: output t % 128, boards 8 (t / 128) ...), so a
// CTA runs 8 warps; the Q heads' outputs reuse the features' region, so
// four CTAs fit on an SM.
__global__ void __launch_bounds__(kHeadThreads, 4) head_kernel(const float *feat, int boards, HeadWeights hw,
                                                               float *logits, float *log_alpha_v, float *log_alpha_q,
                                                               float *alpha_v, float *alpha_q) {
  constexpr int G = kHeadBoards, H = kHeadHalf;
  extern __shared__ __align__(16) float hs[];
  const int A = hw.A, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  float *f = hs;                                    // [81 * 6][G]
  float *hv = f + G * head_shared_floats(A);        // [128][G]
  float *hq = hv + G * kC;
  float *hc = hq + G * kC;
  float *mq = f;                                    // [G][2A], once the features are read
  float *cq = mq + G * 2 * A;                       // [G][A]
  const int e0 = blockIdx.x * G;
  const int nb = min(G, boards - e0);
  const int u = t & (kC - 1), g0 = (t >> 7) * H;    // this thread's output index and first board
  // one (board, cell) per item, boards fastest: a cell's 8 head features
  // are one 32-byte sector
  for (int i = t; i < G * 81; i += kHeadThreads) {
    const int g = i % G, pos = i / G;
    const int y = pos / 9, x = pos % 9;
    float4 lo = make_float4(0.0f, 0.0f, 0.0f, 0.0f), hi = lo;
    if (g < nb) {
      const float4 *src =
          reinterpret_cast<const float4 *>(feat + ((size_t)(e0 + g) * kRowsPerBoard + (y + 1) * 10 + x) * 8);
      lo = src[0];
      hi = src[1];
    }
    float *dst = f + pos * kHeadCh * G + g;
    dst[0 * G] = lo.x;
    dst[1 * G] = lo.y;
    dst[2 * G] = lo.z;
    dst[3 * G] = lo.w;
    dst[4 * G] = hi.x;
    dst[5 * G] = hi.y;
  }
  __syncthreads();
  // policy logits: flatten (y, x, c) of the 2-channel policy features
  for (int a = u; a < A; a += kC) {
    float acc[H];
#pragma unroll
    for (int g = 0; g < H; ++g) acc[g] = hw.policy_b[a];
#pragma unroll 4
    for (int pos = 0; pos < 81; ++pos)
#pragma unroll
      for (int c = 0; c < 2; ++c)
        fma_boards(acc, f + (pos * kHeadCh + c) * G + g0, hw.policy_w[(pos * 2 + c) * A + a]);
#pragma unroll
    for (int g = 0; g < H; ++g)
      if (g0 + g < nb) logits[(size_t)(e0 + g0 + g) * A + a] = acc[g];
  }
  // hidden layers (hidden unit u)
  {
    float v[H], q[H], c[H];
#pragma unroll
    for (int g = 0; g < H; ++g) {
      v[g] = hw.value_b1[u];
      q[g] = hw.qdir_b1[u];
      c[g] = hw.qconc_b1[u];
    }
#pragma unroll 2
    for (int pos = 0; pos < 81; ++pos) {
      const float wv = hw.value_w1[pos * kC + u], wc = hw.qconc_w1[pos * kC + u];
      const float wq0 = hw.qdir_w1[(pos * 2) * kC + u], wq1 = hw.qdir_w1[(pos * 2 + 1) * kC + u];
      const float *fp = f + pos * kHeadCh * G + g0;
      fma_boards(v, fp + 2 * G, wv);
      fma_boards(c, fp + 5 * G, wc);
      fma_boards(q, fp + 3 * G, wq0);
      fma_boards(q, fp + 4 * G, wq1);
    }
#pragma unroll
    for (int g = 0; g < H; ++g) {
      hv[u * G + g0 + g] = fmaxf(v[g], 0.0f);
      hq[u * G + g0 + g] = fmaxf(q[g], 0.0f);
      hc[u * G + g0 + g] = fmaxf(c[g], 0.0f);
    }
  }
  __syncthreads();  // the features are read: mq and cq take their place
  // value head: 2 mean logits + 1 log-concentration, one warp per board
  for (int g = warp; g < nb; g += kHeadThreads / 32) {
    const float *h = hv + g;
    const float m0 = warp_dot128(h, G, hw.value_mean_w, 2, lane) + hw.value_mean_b[0];
    const float m1 = warp_dot128(h, G, hw.value_mean_w + 1, 2, lane) + hw.value_mean_b[1];
    const float cv = warp_dot128(h, G, hw.value_conc_w, 1, lane) + hw.value_conc_b[0];
    if (lane == 0) {
      const int e = e0 + g;
      const float cc = fminf(fmaxf(cv, -80.0f), 80.0f);
      const float mx = fmaxf(m0, m1);
      const float lse = mx + logf(expf(m0 - mx) + expf(m1 - mx));
      log_alpha_v[e * 2] = cc + (m0 - lse);
      log_alpha_v[e * 2 + 1] = cc + (m1 - lse);
      alpha_v[e * 2] = expf(cc + (m0 - lse));
      alpha_v[e * 2 + 1] = expf(cc + (m1 - lse));
    }
  }
  // Q heads: the 2A direction outputs, then the A concentration outputs
  for (int j = u; j < 3 * A; j += kC) {
    const bool dir = j < 2 * A;
    const int jj = dir ? j : j - 2 * A;
    const float *hk = dir ? hq : hc;
    const float *wk = dir ? hw.qdir_w2 + jj : hw.qconc_w2 + jj;
    const int wstride = dir ? 2 * A : A;
    float acc[H];
    const float bias = dir ? hw.qdir_b2[jj] : hw.qconc_b2[jj];
#pragma unroll
    for (int g = 0; g < H; ++g) acc[g] = bias;
#pragma unroll 4
    for (int k = 0; k < kC; ++k) fma_boards(acc, hk + k * G + g0, wk[k * wstride]);
#pragma unroll
    for (int g = 0; g < H; ++g) {
      if (dir)
        mq[(g0 + g) * 2 * A + jj] = acc[g];
      else
        cq[(g0 + g) * A + jj] = acc[g];
    }
  }
  __syncthreads();
  for (int i = t; i < nb * A; i += kHeadThreads) {
    const int g = i / A, a = i % A;
    const float cc = fminf(fmaxf(cq[g * A + a], -80.0f), 80.0f);
    const float q0 = mq[g * 2 * A + 2 * a], q1 = mq[g * 2 * A + 2 * a + 1];
    const float mx = fmaxf(q0, q1);
    const float lse = mx + logf(expf(q0 - mx) + expf(q1 - mx));
    const size_t o = ((size_t)(e0 + g) * A + a) * 2;
    log_alpha_q[o] = cc + (q0 - lse);
    log_alpha_q[o + 1] = cc + (q1 - lse);
    alpha_q[o] = expf(cc + (q0 - lse));
    alpha_q[o + 1] = expf(cc + (q1 - lse));
  }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------

std::atomic<uint64_t> g_tower_launches{0};

// Optional timing of the convolutions: a pair of CUDA events around the
// conv launches of each forward (recorded on the forward's stream), for a
// caller that reports the convolutions' share and throughput inside a
// longer step.  Off unless scacchi_tower_timing enabled it.
struct ConvTiming {
  cudaEvent_t *ev = nullptr;  // [2 * cap]
  int cap = 0, used = 0;
};
ConvTiming g_conv_timing;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2D 16-bit tensor [rows, 128] with 64 x 128 boxes and 128-byte swizzle (the
// copy is type-agnostic; the MMA's instruction descriptor names the format)
bool make_map(CUtensorMap *map, const void *base, uint64_t rows, uint32_t box_rows = kBM) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)kC, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kC * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// in_lo: the lo matrix of split operands (Split), else unused
template <typename T, bool Split>
int launch_conv(const void *in, const void *in_lo, const void *w, void *out0, void *out1, const EpiParams &ep,
                uint64_t rows_alloc, cudaStream_t stream) {
  CUtensorMap m_in, m_in_lo, m_w, m_o0, m_o1;
  const uint64_t w_rows = (uint64_t)9 * kC * (Split && ep.terms == 3 ? 2 : 1);
  if (!make_map(&m_in, in, rows_alloc, kWinBoxRows) || !make_map(&m_w, w, w_rows)) return SCACCHI_ECUDA;
  if (!make_map(&m_in_lo, Split ? in_lo : in, rows_alloc, kWinBoxRows)) return SCACCHI_ECUDA;
  if (!make_map(&m_o0, out0 ? out0 : in, rows_alloc)) return SCACCHI_ECUDA;
  if (!make_map(&m_o1, out1 ? out1 : (out0 ? out0 : in), rows_alloc)) return SCACCHI_ECUDA;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(conv_tc_kernel<T, Split>, cudaFuncAttributeMaxDynamicSharedMemorySize, SmemLayout::kBytes);
    attr = true;
  }
  const int tiles = (int)(rows_alloc / kBM);
  const int pairs = (tiles + 1) / 2;
  const int grid = pairs < num_sms() ? pairs : num_sms();
  conv_tc_kernel<T, Split><<<grid, kThreads, SmemLayout::kBytes, stream>>>(m_in, m_in_lo, m_w, m_o0, m_o1, ep,
                                                                            tiles);
  g_tower_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaPeekAtLastError() == cudaSuccess ? SCACCHI_OK : SCACCHI_ECUDA;
}

bool misaligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; }

}  // namespace

extern "C" {

uint64_t scacchi_tower_rows(int32_t boards) {
  const uint64_t rows = (uint64_t)(boards > 0 ? boards : 0) * kRowsPerBoard;
  return (rows + kBM - 1) / kBM * kBM;
}

size_t scacchi_tower_workspace_bytes(int32_t boards) {
  // split operands: fp32 x + hi/lo of a and h; plain: three 16-bit matrices;
  // then the head features and the stem's subset table
  const uint64_t rows = scacchi_tower_rows(boards);
  return (size_t)rows * kC * (4 + 2 * 4) + (size_t)rows * 8 * 4 + kStemTableBytes;
}

int scacchi_conv3x3(const void *input, const void *weights, const float *bias, int32_t mode, int32_t boards,
                    int32_t fp16, const float *bn_scale, const float *bn_shift, const void *residual,
                    const float *head_w, const float *head_b, void *out0, void *out1, float *head_out,
                    void *stream) {
  if (!input || !weights || !bias || boards < 1 || mode < 0 || mode > 2 || (fp16 != 0 && fp16 != 1))
    return SCACCHI_EINVAL;
  if (mode != kEpiConv1 && (!bn_scale || !bn_shift || !residual)) return SCACCHI_EINVAL;
  if (mode == kEpiHeads && (!head_w || !head_b || !head_out)) return SCACCHI_EINVAL;
  if (mode != kEpiHeads && !out0) return SCACCHI_EINVAL;
  if (mode == kEpiConv2 && !out1) return SCACCHI_EINVAL;
  if ((reinterpret_cast<uintptr_t>(input) | reinterpret_cast<uintptr_t>(weights) |
       reinterpret_cast<uintptr_t>(out0) | reinterpret_cast<uintptr_t>(out1)) & 15u)
    return SCACCHI_EINVAL;
  EpiParams ep;
  ep.mode = mode;
  ep.rows_valid = boards * kRowsPerBoard;
  ep.bias = bias;
  ep.bn_scale = bn_scale;
  ep.bn_shift = bn_shift;
  ep.residual = residual;
  ep.head_w = head_w;
  ep.head_b = head_b;
  ep.head_out = head_out;
  ep.terms = 1;
  ep.x32 = nullptr;
  ep.x32_natural_in = 0;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint64_t rows = scacchi_tower_rows(boards);
  return fp16 ? launch_conv<__half, false>(input, nullptr, weights, out0, out1, ep, rows, st)
              : launch_conv<__nv_bfloat16, false>(input, nullptr, weights, out0, out1, ep, rows, st);
}

int scacchi_conv3x3_split(const void *input, const void *input_lo, const void *weights, const float *bias,
                          int32_t mode, int32_t boards, int32_t fp16, int32_t terms, const float *bn_scale,
                          const float *bn_shift, float *x32, int32_t x32_natural_in, const float *head_w,
                          const float *head_b, void *out_hi, void *out_lo, float *head_out, void *stream) {
  if (!input || !input_lo || !weights || !bias || boards < 1 || mode < 0 || mode > 2 || (fp16 != 0 && fp16 != 1) ||
      terms < 2 || terms > 3 || (x32_natural_in != 0 && x32_natural_in != 1))
    return SCACCHI_EINVAL;
  if (mode != kEpiConv1 && (!bn_scale || !bn_shift || !x32)) return SCACCHI_EINVAL;
  if (mode == kEpiHeads && (!head_w || !head_b || !head_out)) return SCACCHI_EINVAL;
  if (mode != kEpiHeads && (!out_hi || !out_lo)) return SCACCHI_EINVAL;
  if (misaligned16(input) || misaligned16(input_lo) || misaligned16(weights) || misaligned16(out_hi) ||
      misaligned16(out_lo) || misaligned16(x32))
    return SCACCHI_EINVAL;
  EpiParams ep;
  ep.mode = mode;
  ep.rows_valid = boards * kRowsPerBoard;
  ep.terms = terms;
  ep.bias = bias;
  ep.bn_scale = bn_scale;
  ep.bn_shift = bn_shift;
  ep.residual = nullptr;
  ep.x32 = x32;
  ep.x32_natural_in = x32_natural_in;
  ep.head_w = head_w;
  ep.head_b = head_b;
  ep.head_out = head_out;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint64_t rows = scacchi_tower_rows(boards);
  return fp16 ? launch_conv<__half, true>(input, input_lo, weights, out_hi, out_lo, ep, rows, st)
              : launch_conv<__nv_bfloat16, true>(input, input_lo, weights, out_hi, out_lo, ep, rows, st);
}

int scacchi_tower_forward(const scacchi_tower_weights *w, const float *obs, int32_t boards, void *workspace,
                          float *logits, float *log_alpha_v, float *log_alpha_q, float *alpha_v, float *alpha_q,
                          void *stream) {
  if (!w || !obs || boards < 1 || !workspace || !logits || !log_alpha_v || !log_alpha_q || !alpha_v || !alpha_q)
    return SCACCHI_EINVAL;
  if (w->channels != kC || w->height != 9 || w->width != 9 || w->num_blocks < 1 || w->in_planes < 1 ||
      w->in_planes > 16 || w->num_actions < 1 || w->num_actions > 256)
    return SCACCHI_EINVAL;
  if ((w->fp16 != 0 && w->fp16 != 1) || w->terms < 1 || w->terms > 3) return SCACCHI_EINVAL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint64_t rows = scacchi_tower_rows(boards);
  const bool split = w->terms > 1;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  // plain: x, a, h 16-bit; split: x fp32, then the hi/lo pairs of a and h
  float *x32 = split ? reinterpret_cast<float *>(ws) : nullptr;
  uint16_t *x = split ? nullptr : reinterpret_cast<uint16_t *>(ws);
  uint16_t *a = split ? reinterpret_cast<uint16_t *>(x32 + rows * kC) : x + rows * kC;
  uint16_t *a_lo = split ? a + rows * kC : nullptr;
  uint16_t *h = split ? a_lo + rows * kC : a + rows * kC;
  uint16_t *h_lo = split ? h + rows * kC : nullptr;
  float *feat = reinterpret_cast<float *>((split ? h_lo : h) + rows * kC);
  float *stem_table = feat + rows * 8;  // 16-byte aligned: rows is a multiple of 128
  // rows past the last board stay zero (they are padding for the last tile)
  const uint64_t used = (uint64_t)boards * kRowsPerBoard;
  if (rows > used) {
    if (split) {
      cudaMemsetAsync(x32 + used * kC, 0, (rows - used) * kC * 4, st);
      cudaMemsetAsync(a_lo + used * kC, 0, (rows - used) * kC * 2, st);
    } else {
      cudaMemsetAsync(x + used * kC, 0, (rows - used) * kC * 2, st);
    }
    cudaMemsetAsync(a + used * kC, 0, (rows - used) * kC * 2, st);
  }
  const size_t smem = stem_smem_bytes(w->in_planes);
  const int stem_grid = (boards + kStemBoards - 1) / kStemBoards;
  if (w->in_planes <= 4) {
    stem_table_kernel<<<(9 * kStemSubsets * kC + 255) / 256, 256, 0, st>>>(w->in_planes, w->stem_w, stem_table);
    g_tower_launches.fetch_add(1, std::memory_order_relaxed);
  }
#define SCACCHI_STEM(TT, SPLIT)                                                                                     \
  stem_kernel<TT, SPLIT><<<stem_grid, kStemThreads, smem, st>>>(                                                   \
      obs, boards, w->in_planes, w->stem_w, stem_table, w->stem_b, w->bn_scale, w->bn_shift,                      \
      reinterpret_cast<TT *>(x), reinterpret_cast<TT *>(a), x32, reinterpret_cast<TT *>(a_lo))
  if (w->fp16) {
    if (split) SCACCHI_STEM(__half, true);
    else SCACCHI_STEM(__half, false);
  } else {
    if (split) SCACCHI_STEM(__nv_bfloat16, true);
    else SCACCHI_STEM(__nv_bfloat16, false);
  }
#undef SCACCHI_STEM
  g_tower_launches.fetch_add(1, std::memory_order_relaxed);
  // per layer: [terms == 3 ? 2 : 1][9 taps][128 out][128 in]
  const size_t conv_elems = (size_t)9 * kC * kC * (w->terms == 3 ? 2 : 1);
  const int timed = g_conv_timing.used < g_conv_timing.cap ? g_conv_timing.used++ : -1;
  if (timed >= 0) cudaEventRecord(g_conv_timing.ev[2 * timed], st);
  for (int blk = 0; blk < w->num_blocks; ++blk) {
    const uint16_t *w1 = w->conv_w + (size_t)(2 * blk) * conv_elems;
    const uint16_t *w2 = w->conv_w + (size_t)(2 * blk + 1) * conv_elems;
    const bool last = blk == w->num_blocks - 1;
    const int mode2 = last ? kEpiHeads : kEpiConv2;
    const float *s2 = w->bn_scale + (blk + 1) * kC, *t2 = w->bn_shift + (blk + 1) * kC;
    int rc;
    if (split) {
      rc = scacchi_conv3x3_split(a, a_lo, w1, w->conv_b + (2 * blk) * kC, kEpiConv1, boards, w->fp16, w->terms,
                                 nullptr, nullptr, nullptr, 0, nullptr, nullptr, h, h_lo, nullptr, stream);
      if (rc) return rc;
      // the stem leaves x32 in the natural channel order; the first block's
      // conv2 reads it so and writes the x32_slot order the others use
      rc = scacchi_conv3x3_split(h, h_lo, w2, w->conv_b + (2 * blk + 1) * kC, mode2, boards, w->fp16, w->terms, s2,
                                 t2, x32, blk == 0 ? 1 : 0, w->head_w, w->head_b, last ? nullptr : a,
                                 last ? nullptr : a_lo, feat, stream);
    } else {
      rc = scacchi_conv3x3(a, w1, w->conv_b + (2 * blk) * kC, kEpiConv1, boards, w->fp16, nullptr, nullptr, nullptr,
                           nullptr, nullptr, h, nullptr, nullptr, stream);
      if (rc) return rc;
      rc = scacchi_conv3x3(h, w2, w->conv_b + (2 * blk + 1) * kC, mode2, boards, w->fp16, s2, t2, x, w->head_w,
                           w->head_b, last ? nullptr : x, last ? nullptr : a, feat, stream);
    }
    if (rc) return rc;
  }
  if (timed >= 0) cudaEventRecord(g_conv_timing.ev[2 * timed + 1], st);
  HeadWeights hw;
  hw.A = w->num_actions;
  hw.policy_w = w->policy_w;
  hw.policy_b = w->policy_b;
  hw.value_w1 = w->value_w1;
  hw.value_b1 = w->value_b1;
  hw.value_mean_w = w->value_mean_w;
  hw.value_mean_b = w->value_mean_b;
  hw.value_conc_w = w->value_conc_w;
  hw.value_conc_b = w->value_conc_b;
  hw.qdir_w1 = w->qdir_w1;
  hw.qdir_b1 = w->qdir_b1;
  hw.qdir_w2 = w->qdir_w2;
  hw.qdir_b2 = w->qdir_b2;
  hw.qconc_w1 = w->qconc_w1;
  hw.qconc_b1 = w->qconc_b1;
  hw.qconc_w2 = w->qconc_w2;
  hw.qconc_b2 = w->qconc_b2;
  const size_t head_smem = head_smem_bytes(hw.A);
  static std::atomic<size_t> head_attr{0};
  if (head_smem > 48 * 1024 && head_attr.load() < head_smem) {
    cudaFuncSetAttribute(head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)head_smem);
    head_attr.store(head_smem);
  }
  head_kernel<<<(boards + kHeadBoards - 1) / kHeadBoards, kHeadThreads, head_smem, st>>>(
      feat, boards, hw, logits, log_alpha_v, log_alpha_q, alpha_v, alpha_q);
  g_tower_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaPeekAtLastError() == cudaSuccess ? SCACCHI_OK : SCACCHI_ECUDA;
}

int scacchi_tower_error(uint32_t *flags) {
  if (!flags) return SCACCHI_EINVAL;
  uint32_t v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_tower_error, sizeof(v)) != cudaSuccess) return SCACCHI_ECUDA;
  if (cudaMemcpyToSymbol(g_tower_error, &zero, sizeof(zero)) != cudaSuccess) return SCACCHI_ECUDA;
  *flags = v;
  return SCACCHI_OK;
}

uint64_t scacchi_tower_launch_count(void) { return g_tower_launches.load(std::memory_order_relaxed); }

int scacchi_tower_timing(int32_t max_forwards) {
  if (max_forwards < 0) return SCACCHI_EINVAL;
  ConvTiming &t = g_conv_timing;
  for (int i = 0; i < 2 * t.cap; ++i) cudaEventDestroy(t.ev[i]);
  delete[] t.ev;
  t = ConvTiming();
  if (max_forwards == 0) return SCACCHI_OK;
  t.ev = new cudaEvent_t[2 * (size_t)max_forwards];
  for (int i = 0; i < 2 * max_forwards; ++i) {
    if (cudaEventCreate(&t.ev[i]) != cudaSuccess) {
      for (int j = 0; j < i; ++j) cudaEventDestroy(t.ev[j]);
      delete[] t.ev;
      t = ConvTiming();
      return SCACCHI_ECUDA;
    }
  }
  t.cap = max_forwards;
  return SCACCHI_OK;
}

int scacchi_tower_timing_read(float *conv_ms, int32_t *forwards) {
  if (!conv_ms || !forwards) return SCACCHI_EINVAL;
  ConvTiming &t = g_conv_timing;
  float total = 0.0f;
  for (int i = 0; i < t.used; ++i) {
    float ms = 0.0f;
    if (cudaEventSynchronize(t.ev[2 * i + 1]) != cudaSuccess ||
        cudaEventElapsedTime(&ms, t.ev[2 * i], t.ev[2 * i + 1]) != cudaSuccess)
      return SCACCHI_ECUDA;
    total += ms;
  }
  *conv_ms = total;
  *forwards = t.used;
  t.used = 0;
  return SCACCHI_OK;
}

}  // extern "C"
