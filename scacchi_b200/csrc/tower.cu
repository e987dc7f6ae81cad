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
// conv_tc_kernel: persistent (one CTA per SM), warp-specialised
//   warp 0      TMA producer: A (128 rows x 64 ch) + B (128 out x 64 in) per
//               K block, 4-stage mbarrier ring
//   warp 1      TMEM allocator and MMA issuer (one thread):
//               tcgen05.mma.cta_group::1.kind::f16, M = N = 128, K = 16,
//               bf16 x bf16 -> fp32 accumulated in TMEM (two 128-column
//               accumulators so the epilogue of tile i overlaps tile i+1)
//   warps 2-5   epilogue: tcgen05.ld 32x32b, fused bias / folded BatchNorm /
//               ReLU / residual / next block's BN-ReLU, bf16 into
//               128B-swizzled shared memory, TMA store; the last layer
//               instead computes the heads' 1x1 convolutions per row.
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
constexpr int kBM = 128;         // rows per tile
constexpr int kBK = 64;          // channels per K block (128 bytes of bf16)
constexpr int kKBlocks = 18;     // 9 taps x 2 channel blocks
constexpr int kStages = 4;
constexpr int kTileBytes = kBM * kBK * 2;  // 16 KB
constexpr int kStageBytes = 2 * kTileBytes;
constexpr int kThreads = 192;
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

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (leading offset unused for swizzled K-major layouts)
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;             // leading byte offset (16 B units)
  d |= (uint64_t)(1024u >> 4) << 32;   // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1u << 46;             // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;             // SWIZZLE_128B
  return d;
}

// instruction descriptor (idesc_for below): D f32 (bits 4-5), A/B format
// (bits 7-9 / 10-12: 0 f16, 1 bf16), K-major A and B, N >> 3 at bit 17,
// M >> 4 at bit 24; here M = N = 128

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

template <typename T>
__host__ __device__ constexpr uint32_t idesc_for() {
  return (1u << 4) | (F16Traits<T>::kFormat << 7) | (F16Traits<T>::kFormat << 10) | ((128u >> 3) << 17) |
         ((128u >> 4) << 24);
}

// ---------------------------------------------------------------------------
// convolution kernel
// ---------------------------------------------------------------------------

enum EpiMode : int { kEpiConv1 = 0, kEpiConv2 = 1, kEpiHeads = 2 };

struct EpiParams {
  int mode;
  int rows_valid;            // E * 100; rows at or above are padding
  const float *bias;         // [128] (BatchNorm after conv1 folded in)
  const float *bn_scale;     // conv2: next block's BN1 (or the final BN), per channel
  const float *bn_shift;
  const void *residual;      // conv2 / heads: x of the block input, [rows, 128] 16-bit
  const float *head_w;       // heads: [6][128] 1x1 conv weights (head BN folded)
  const float *head_b;       // [6]
  float *head_out;           // heads: [rows, 8] f32
};

struct SmemLayout {
  static constexpr int kStagesOff = 0;
  static constexpr int kOutOff = kStages * kStageBytes;               // 2 outputs x 2 halves x 16 KB
  static constexpr int kParamOff = kOutOff + 4 * kTileBytes;           // floats
  static constexpr int kParamFloats = 3 * kC + kHeadCh * kC + 8;
  static constexpr int kBarOff = kParamOff + kParamFloats * 4;
  static constexpr int kBytes = kBarOff + 8 * (2 * kStages + 4) + 16 + 1024;  // + alignment slack

};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) conv_tc_kernel(const __grid_constant__ CUtensorMap tm_in,
                                                              const __grid_constant__ CUtensorMap tm_w,
                                                              const __grid_constant__ CUtensorMap tm_out0,
                                                              const __grid_constant__ CUtensorMap tm_out1,
                                                              EpiParams ep, int num_tiles) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float *prm = reinterpret_cast<float *>(smem + SmemLayout::kParamOff);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + SmemLayout::kBarOff);
  uint64_t *empty = full + kStages;
  uint64_t *acc_full = empty + kStages;
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
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;  // per stage: issued?, parity of the last load
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        const int row0 = tile * kBM;
        for (int kb = 0; kb < kKBlocks; ++kb) {
          const int tap = kb >> 1, cb = kb & 1;
          const int off = (tap / 3 - 1) * 10 + (tap % 3 - 1);
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) break;
          uint8_t *sa = smem + SmemLayout::kStagesOff + stage * kStageBytes;
          mbar_expect_tx(&full[stage], kStageBytes);
          tma_load_2d(sa, &tm_in, &full[stage], cb * kBK, row0 + off);
          tma_load_2d(sa + kTileBytes, &tm_w, &full[stage], cb * kBK, tap * kC);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // every load issued into shared memory lands before the CTA may exit
      for (int s = 0; s < kStages; ++s) {
        if (!(issued_mask >> s & 1u)) continue;
        mbar_drain(&full[s], issued_parity >> s & 1u);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * kC);
        bool ok = true;
        for (int kb = 0; kb < kKBlocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + SmemLayout::kStagesOff + stage * kStageBytes);
          const uint32_t sb = sa + kTileBytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t adesc = smem_desc_sw128(sa + k * 32);
            const uint64_t bdesc = smem_desc_sw128(sb + k * 32);
            umma_f16(d, adesc, bdesc, idesc_for<T>(), (kb | k) != 0);
          }
          umma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2-5) ----------------
    const int quad = warp & 3;              // TMEM lanes this warp may access
    const int row_in_tile = quad * 32 + lane;
    const int et = threadIdx.x - 64;        // 0..127
    uint8_t *out0 = smem + SmemLayout::kOutOff;
    uint8_t *out1 = out0 + 2 * kTileBytes;
    volatile int *go = abort_flag + 1;  // elected thread's verdict for the tile
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      // one thread waits (bounded) and broadcasts, so the 128 threads agree
      if (et == 0) {
        const bool ok = !*abort_flag && mbar_wait(&acc_full[acc], acc_phase, abort_flag);
        // staging buffers must be free (previous tile's TMA store read them)
        tma_store_wait_read();
        *go = ok ? 1 : 0;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (!*go) break;
      asm volatile("bar.sync 1, 128;" ::: "memory");  // everyone read `go` before it changes
      tc_fence_after();
      const int r = tile * kBM + row_in_tile;
      const int p = r % kRowsPerBoard;
      const bool real = r < ep.rows_valid && p >= 10 && (p % 10) != 9;
      float head[kHeadCh];
#pragma unroll
      for (int h = 0; h < kHeadCh; ++h) head[h] = 0.0f;
      for (int ch = 0; ch < 4; ++ch) {
        float v[32];
        tmem_ld32(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * kC + ch * 32), v);
        float res[32];
        if (ep.mode != kEpiConv1) {
          const uint4 *src =
              reinterpret_cast<const uint4 *>(static_cast<const T *>(ep.residual) + (size_t)r * kC + ch * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 u = real ? src[q] : make_uint4(0, 0, 0, 0);
            const T *hb = reinterpret_cast<const T *>(&u);
#pragma unroll
            for (int e = 0; e < 8; ++e) res[q * 8 + e] = F16Traits<T>::to_f(hb[e]);
          }
        }
        uint32_t pk0[16], pk1[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float o0[2], o1[2];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int n = ch * 32 + i + j;
            float y = v[i + j] + prm[n];
            if (ep.mode == kEpiConv1) {
              y = real ? fmaxf(y, 0.0f) : 0.0f;
              o0[j] = y;
              o1[j] = 0.0f;
            } else {
              // residual stream stored in the 16-bit type like the reference's bf16 model
              const float xn = F16Traits<T>::to_f(F16Traits<T>::from_f(y + res[i + j]));
              const float a = fmaxf(fmaf(xn, prm[kC + n], prm[2 * kC + n]), 0.0f);
              o0[j] = real ? xn : 0.0f;
              o1[j] = real ? F16Traits<T>::to_f(F16Traits<T>::from_f(a)) : 0.0f;
              if (ep.mode == kEpiHeads) {
#pragma unroll
                for (int h = 0; h < kHeadCh; ++h) head[h] = fmaf(o1[j], prm[3 * kC + h * kC + n], head[h]);
              }
            }
          }
          pk0[i / 2] = F16Traits<T>::pack(o0[0], o0[1]);
          pk1[i / 2] = F16Traits<T>::pack(o1[0], o1[1]);
        }
        if (ep.mode != kEpiHeads) {
          // 32 channels = four 16-byte chunks of the 64-channel half `ch / 2`
          uint8_t *h0 = out0 + (ch >> 1) * kTileBytes;
          uint8_t *h1 = out1 + (ch >> 1) * kTileBytes;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int chunk = (ch & 1) * 4 + q;
            *reinterpret_cast<uint4 *>(h0 + swz(row_in_tile, chunk)) =
                make_uint4(pk0[4 * q], pk0[4 * q + 1], pk0[4 * q + 2], pk0[4 * q + 3]);
            if (ep.mode == kEpiConv2)
              *reinterpret_cast<uint4 *>(h1 + swz(row_in_tile, chunk)) =
                  make_uint4(pk1[4 * q], pk1[4 * q + 1], pk1[4 * q + 2], pk1[4 * q + 3]);
          }
        }
      }
      // the accumulator can be reused by the MMA warp
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
      if (ep.mode == kEpiHeads) {
        if (r < ep.rows_valid) {
          float4 *dst = reinterpret_cast<float4 *>(ep.head_out + (size_t)r * 8);
          float hb[kHeadCh];
#pragma unroll
          for (int h = 0; h < kHeadCh; ++h) hb[h] = real ? fmaxf(head[h] + prm[3 * kC + kHeadCh * kC + h], 0.0f) : 0.0f;
          dst[0] = make_float4(hb[0], hb[1], hb[2], hb[3]);
          dst[1] = make_float4(hb[4], hb[5], 0.0f, 0.0f);
        }
        continue;
      }
      fence_proxy_async();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (et == 0) {
        const int row0 = tile * kBM;
        tma_store_2d(&tm_out0, out0, 0, row0);
        tma_store_2d(&tm_out0, out0 + kTileBytes, kBK, row0);
        if (ep.mode == kEpiConv2) {
          tma_store_2d(&tm_out1, out1, 0, row0);
          tma_store_2d(&tm_out1, out1 + kTileBytes, kBK, row0);
        }
        tma_store_commit();
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
    tmem_dealloc(tmem_base, 256);
  }
}

// ---------------------------------------------------------------------------
// stem: conv3x3 in_planes -> 128 (+ bias), then BN1 of block 0 and ReLU
// ---------------------------------------------------------------------------

template <typename T>
__global__ void stem_kernel(const float *obs, int in_planes, const float *w, const float *b, const float *s1,
                            const float *t1, T *x, T *a) {
  extern __shared__ float sm[];
  const int e = blockIdx.x, n = threadIdx.x;
  float *so = sm;                       // [9*9*in_planes]
  float *sw = sm + 81 * in_planes;      // [9 * in_planes][128]
  for (int i = n; i < 81 * in_planes; i += blockDim.x) so[i] = obs[(size_t)e * 81 * in_planes + i];
  for (int i = n; i < 9 * in_planes * kC; i += blockDim.x) sw[i] = w[i];
  __syncthreads();
  const float bias = b[n], sc = s1[n], sh = t1[n];
  for (int p = 0; p < kRowsPerBoard; ++p) {
    const int yp = p / 10, xp = p % 10;
    const bool real = yp >= 1 && xp <= 8;
    float acc = bias;
    if (real) {
      const int y = yp - 1, xx = xp;
      for (int ky = 0; ky < 3; ++ky) {
        const int iy = y + ky - 1;
        if (iy < 0 || iy >= 9) continue;
        for (int kx = 0; kx < 3; ++kx) {
          const int ix = xx + kx - 1;
          if (ix < 0 || ix >= 9) continue;
          const float *o = so + (iy * 9 + ix) * in_planes;
          const float *wt = sw + ((ky * 3 + kx) * in_planes) * kC + n;
          for (int c = 0; c < in_planes; ++c) acc = fmaf(o[c], wt[c * kC], acc);
        }
      }
    }
    const size_t r = (size_t)e * kRowsPerBoard + p;
    const T xb = F16Traits<T>::from_f(real ? acc : 0.0f);
    x[r * kC + n] = xb;
    const float av = fmaxf(fmaf(F16Traits<T>::to_f(xb), sc, sh), 0.0f);
    a[r * kC + n] = F16Traits<T>::from_f(real ? av : 0.0f);
  }
}

// ---------------------------------------------------------------------------
// heads: per board, the linears on the 1x1-conv features, then
// dirichlet_from_logits (network.py:150-212, log-concentration heads)
// ---------------------------------------------------------------------------

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

__device__ __forceinline__ float block_sum128(float v, float *red) {
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  return red[0] + red[1] + red[2] + red[3];
}

__global__ void __launch_bounds__(128) head_kernel(const float *feat, HeadWeights hw, float *logits,
                                                   float *log_alpha_v, float *log_alpha_q, float *alpha_v,
                                                   float *alpha_q) {
  __shared__ float f[81 * kHeadCh];
  __shared__ float hv[kC], hq[kC], hc[kC];
  __shared__ float mq[2 * 128], cq[128];
  __shared__ float red[8];
  const int e = blockIdx.x, t = threadIdx.x, A = hw.A;
  for (int i = t; i < 81 * kHeadCh; i += 128) {
    const int pos = i / kHeadCh, c = i % kHeadCh;
    const int y = pos / 9, x = pos % 9;
    f[i] = feat[((size_t)e * kRowsPerBoard + (y + 1) * 10 + x) * 8 + c];
  }
  __syncthreads();
  // policy logits: flatten (y, x, c) of the 2-channel policy features
  for (int a = t; a < A; a += 128) {
    float acc = hw.policy_b[a];
    for (int pos = 0; pos < 81; ++pos)
      for (int c = 0; c < 2; ++c) acc = fmaf(f[pos * kHeadCh + c], hw.policy_w[(pos * 2 + c) * A + a], acc);
    logits[(size_t)e * A + a] = acc;
  }
  // hidden layers (thread t = hidden unit t)
  {
    float v = hw.value_b1[t], q = hw.qdir_b1[t], c = hw.qconc_b1[t];
    for (int pos = 0; pos < 81; ++pos) {
      v = fmaf(f[pos * kHeadCh + 2], hw.value_w1[pos * kC + t], v);
      c = fmaf(f[pos * kHeadCh + 5], hw.qconc_w1[pos * kC + t], c);
      q = fmaf(f[pos * kHeadCh + 3], hw.qdir_w1[(pos * 2) * kC + t], q);
      q = fmaf(f[pos * kHeadCh + 4], hw.qdir_w1[(pos * 2 + 1) * kC + t], q);
    }
    hv[t] = fmaxf(v, 0.0f);
    hq[t] = fmaxf(q, 0.0f);
    hc[t] = fmaxf(c, 0.0f);
  }
  __syncthreads();
  // value head: 2 mean logits + 1 log-concentration
  const float m0 = block_sum128(hv[t] * hw.value_mean_w[t * 2], red) + hw.value_mean_b[0];
  const float m1 = block_sum128(hv[t] * hw.value_mean_w[t * 2 + 1], red) + hw.value_mean_b[1];
  const float cv = block_sum128(hv[t] * hw.value_conc_w[t], red) + hw.value_conc_b[0];
  if (t == 0) {
    const float cc = fminf(fmaxf(cv, -80.0f), 80.0f);
    const float mx = fmaxf(m0, m1);
    const float lse = mx + logf(expf(m0 - mx) + expf(m1 - mx));
    log_alpha_v[e * 2] = cc + (m0 - lse);
    log_alpha_v[e * 2 + 1] = cc + (m1 - lse);
    alpha_v[e * 2] = expf(cc + (m0 - lse));
    alpha_v[e * 2 + 1] = expf(cc + (m1 - lse));
  }
  // Q heads
  for (int j = t; j < 2 * A; j += 128) {
    float acc = hw.qdir_b2[j];
    for (int k = 0; k < kC; ++k) acc = fmaf(hq[k], hw.qdir_w2[k * 2 * A + j], acc);
    mq[j] = acc;
  }
  for (int a = t; a < A; a += 128) {
    float acc = hw.qconc_b2[a];
    for (int k = 0; k < kC; ++k) acc = fmaf(hc[k], hw.qconc_w2[k * A + a], acc);
    cq[a] = acc;
  }
  __syncthreads();
  for (int a = t; a < A; a += 128) {
    const float cc = fminf(fmaxf(cq[a], -80.0f), 80.0f);
    const float q0 = mq[2 * a], q1 = mq[2 * a + 1];
    const float mx = fmaxf(q0, q1);
    const float lse = mx + logf(expf(q0 - mx) + expf(q1 - mx));
    const size_t o = ((size_t)e * A + a) * 2;
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
bool make_map(CUtensorMap *map, const void *base, uint64_t rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)kC, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kC * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
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

template <typename T>
int launch_conv(const void *in, const void *w, void *out0, void *out1, const EpiParams &ep, uint64_t rows_alloc,
                cudaStream_t stream) {
  CUtensorMap m_in, m_w, m_o0, m_o1;
  if (!make_map(&m_in, in, rows_alloc) || !make_map(&m_w, w, 9 * kC)) return SCACCHI_ECUDA;
  if (!make_map(&m_o0, out0 ? out0 : in, rows_alloc)) return SCACCHI_ECUDA;
  if (!make_map(&m_o1, out1 ? out1 : (out0 ? out0 : in), rows_alloc)) return SCACCHI_ECUDA;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(conv_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, SmemLayout::kBytes);
    attr = true;
  }
  const int tiles = (int)(rows_alloc / kBM);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  conv_tc_kernel<T><<<grid, kThreads, SmemLayout::kBytes, stream>>>(m_in, m_w, m_o0, m_o1, ep, tiles);
  g_tower_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaPeekAtLastError() == cudaSuccess ? SCACCHI_OK : SCACCHI_ECUDA;
}

}  // namespace

extern "C" {

uint64_t scacchi_tower_rows(int32_t boards) {
  const uint64_t rows = (uint64_t)(boards > 0 ? boards : 0) * kRowsPerBoard;
  return (rows + kBM - 1) / kBM * kBM;
}

size_t scacchi_tower_workspace_bytes(int32_t boards) {
  const uint64_t rows = scacchi_tower_rows(boards);
  return (size_t)rows * kC * 2 * 3 + (size_t)rows * 8 * 4;
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
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint64_t rows = scacchi_tower_rows(boards);
  return fp16 ? launch_conv<__half>(input, weights, out0, out1, ep, rows, st)
              : launch_conv<__nv_bfloat16>(input, weights, out0, out1, ep, rows, st);
}

int scacchi_tower_forward(const scacchi_tower_weights *w, const float *obs, int32_t boards, void *workspace,
                          float *logits, float *log_alpha_v, float *log_alpha_q, float *alpha_v, float *alpha_q,
                          void *stream) {
  if (!w || !obs || boards < 1 || !workspace || !logits || !log_alpha_v || !log_alpha_q || !alpha_v || !alpha_q)
    return SCACCHI_EINVAL;
  if (w->channels != kC || w->height != 9 || w->width != 9 || w->num_blocks < 1 || w->in_planes < 1 ||
      w->in_planes > 16 || w->num_actions < 1 || w->num_actions > 256)
    return SCACCHI_EINVAL;
  if (w->fp16 != 0 && w->fp16 != 1) return SCACCHI_EINVAL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint64_t rows = scacchi_tower_rows(boards);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  uint16_t *x = reinterpret_cast<uint16_t *>(ws);
  uint16_t *a = x + rows * kC;
  uint16_t *h = a + rows * kC;
  float *feat = reinterpret_cast<float *>(h + rows * kC);
  // rows past the last board stay zero (they are padding for the last tile)
  const uint64_t used = (uint64_t)boards * kRowsPerBoard;
  if (rows > used) {
    cudaMemsetAsync(x + used * kC, 0, (rows - used) * kC * 2, st);
    cudaMemsetAsync(a + used * kC, 0, (rows - used) * kC * 2, st);
  }
  const size_t smem = (size_t)(81 * w->in_planes + 9 * w->in_planes * kC) * sizeof(float);
  if (w->fp16)
    stem_kernel<__half><<<boards, kC, smem, st>>>(obs, w->in_planes, w->stem_w, w->stem_b, w->bn_scale, w->bn_shift,
                                                  reinterpret_cast<__half *>(x), reinterpret_cast<__half *>(a));
  else
    stem_kernel<__nv_bfloat16><<<boards, kC, smem, st>>>(obs, w->in_planes, w->stem_w, w->stem_b, w->bn_scale,
                                                         w->bn_shift, reinterpret_cast<__nv_bfloat16 *>(x),
                                                         reinterpret_cast<__nv_bfloat16 *>(a));
  g_tower_launches.fetch_add(1, std::memory_order_relaxed);
  const size_t conv_elems = (size_t)9 * kC * kC;
  for (int blk = 0; blk < w->num_blocks; ++blk) {
    const uint16_t *w1 = w->conv_w + (size_t)(2 * blk) * conv_elems;
    const uint16_t *w2 = w->conv_w + (size_t)(2 * blk + 1) * conv_elems;
    int rc = scacchi_conv3x3(a, w1, w->conv_b + (2 * blk) * kC, kEpiConv1, boards, w->fp16, nullptr, nullptr,
                             nullptr, nullptr, nullptr, h, nullptr, nullptr, stream);
    if (rc) return rc;
    const bool last = blk == w->num_blocks - 1;
    rc = scacchi_conv3x3(h, w2, w->conv_b + (2 * blk + 1) * kC, last ? kEpiHeads : kEpiConv2, boards, w->fp16,
                         w->bn_scale + (blk + 1) * kC, w->bn_shift + (blk + 1) * kC, x, w->head_w, w->head_b,
                         last ? nullptr : x, last ? nullptr : a, feat, stream);
    if (rc) return rc;
  }
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
  head_kernel<<<boards, 128, 0, st>>>(feat, hw, logits, log_alpha_v, log_alpha_q, alpha_v, alpha_q);
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

}  // extern "C"
