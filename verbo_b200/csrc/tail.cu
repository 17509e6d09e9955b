// Kernels of the logits producer tail (src/session.cpp:163-169).
//
// tail_norm_kernel      one CTA per hidden row: rmsnorm (src/session.cpp:14-19)
//                       and, for quantised heads, quant_act (src/kernels.cpp:106),
//                       written as the head kernel's activation blocks;
// tail_head_q_kernel    Q8 / Q4 heads: a producer warp streams tile-major
//                       head blocks (and activation blocks) into a ring of
//                       shared-memory stages with bulk copies; eight consumer
//                       warps run one int8 m16n8k32 tensor-core MMA per
//                       32-element block and apply the block's fp32 scale in
//                       that MMA's epilogue (dot_q8 / dot_q4,
//                       src/kernels.cpp:576-600);
// tail_head_f32_kernel  F32 heads: the same ring over a tile-major fp32 head,
//                       one vocab row per consumer thread (dot_f32,
//                       src/kernels.cpp:570-574);
// tail_head_tc_kernel   Q8 heads with more than 32 tokens, on request
//                       (VERBO_CUDA_TAIL_TCGEN05=1): tcgen05.mma kind::i8 per
//                       block into tensor memory, the same epilogue in
//                       epilogue warps.  Bit-identical, but slower than the
//                       mma.sync kernel here: both are bound by the
//                       epilogue's fp32 work per block, and the tensor-memory
//                       round trip of every block adds to it.
//
// Every rounding step is the reference scalar build's, in its order: the sum
// of squares runs sequentially, products and sums are rounded separately
// where the reference rounds them separately (__fmul_rn / __fadd_rn are never
// contracted), and the block accumulate is the one FMA the reference's build
// forms, r = fma(scale_w * scale_x, float(block sum), r), in block order.
#include <cuda_fp16.h>

#include <cstdlib>
#include <cstring>

#include "device.cuh"
#include "tail.cuh"

namespace vb {
namespace {

__device__ unsigned int g_tail_status;

constexpr int kMagicBits = 0x4B400000;  // bits of 1.5 * 2^23
constexpr float kMagic = 12582912.0f;   // 1.5 * 2^23
constexpr int kConsumers = 8;           // consumer warps of the head kernel
constexpr int kHeadThreads = (kConsumers + 1) * 32;
constexpr int kL2Ahead = 10;            // head blocks a CTA prefetches into L2 before waiting for the norm

// ---------------------------------------------------------------- norm ----
// Thread 0 sums the squares in index order (the reference's loop), reading
// the staged row 32 values at a time so that only the chain of adds is
// serial; the CTA then normalises, and each warp quantises one 32-block at a
// time.  CTAs past the last row write the zero padding of the token tile.
__global__ void __launch_bounds__(kTailThreads) tail_norm_kernel(TailHead h, TailArgs a) {
  // Launched with programmatic serialization: wait for the preceding grid (it
  // may write x), then let the head kernel start streaming weights; it waits
  // for this grid before it requests the activations.
  grid_wait();
  grid_release();
  extern __shared__ __align__(16) float xr[];  // the row, then the norm weights: 2 x dim floats
  float* nw = xr + h.dim;
  __shared__ float s_r;
  const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nbp = h.dimp / kTailBlk;
  const int ncol = a.n_pad / a.nt, ct = row / a.nt, c = row % a.nt;
  const size_t actb = static_cast<size_t>(a.nt) * (kTailChunk + 16);
  if (row >= a.n && h.dtype == kTailF32) {  // padding token of an fp32 head
    for (int i = threadIdx.x; i < h.dim; i += kTailThreads)
      a.xb[((static_cast<size_t>(i >> 5) * ncol + ct) * 32 + (i & 31)) * a.nt + c] = 0.0f;
    return;
  }
  if (row >= a.n) {  // padding token of a quantised head
    for (int b = warp; b < nbp; b += kTailThreads / 32) {
      unsigned char* blk = a.act + (static_cast<size_t>(b >> 2) * ncol + ct) * actb;
      blk[c * kTailChunk + (b & 3) * 32 + lane] = 0;
      if (lane == 0) reinterpret_cast<float*>(blk + a.nt * kTailChunk)[(b & 3) * a.nt + c] = 0.0f;
    }
    return;
  }
  const float* x = a.x + static_cast<long long>(row) * a.ldx;
  for (int i = threadIdx.x; i < h.dim; i += kTailThreads) {
    xr[i] = x[i];
    nw[i] = h.norm[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float ss = 0.0f;
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = *reinterpret_cast<const float4*>(xr + 4 * j);
    for (int i = 0; i < h.dim; i += 32) {  // dim is a multiple of 32
      // the next 32 values load while these 32 are added
      const int nx = i + 32 < h.dim ? i + 32 : i;
      float4 w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = *reinterpret_cast<const float4*>(xr + nx + 4 * j);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        ss = __fadd_rn(ss, __fmul_rn(v[j].x, v[j].x));
        ss = __fadd_rn(ss, __fmul_rn(v[j].y, v[j].y));
        ss = __fadd_rn(ss, __fmul_rn(v[j].z, v[j].z));
        ss = __fadd_rn(ss, __fmul_rn(v[j].w, v[j].w));
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = w[j];
    }
    s_r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(h.dim)), h.eps)));
  }
  __syncthreads();
  const float r = s_r;
  if (h.dtype == kTailF32) {  // activation blocks [dim / 32][token tiles][32][nt]
    for (int i = threadIdx.x; i < h.dim; i += kTailThreads)
      a.xb[((static_cast<size_t>(i >> 5) * ncol + ct) * 32 + (i & 31)) * a.nt + c] =
          __fmul_rn(nw[i], __fmul_rn(xr[i], r));
    return;
  }
  // four blocks per warp at a time, so that their shuffle and division chains overlap
  constexpr int W = kTailThreads / 32;
  for (int b0 = warp; b0 < nbp; b0 += 4 * W) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = b0 + j * W;
      if (b < nbp) {
        const int i = b * kTailBlk + lane;
        const float v = i < h.dim ? __fmul_rn(nw[i], __fmul_rn(xr[i], r)) : 0.0f;
        // std::max(amax, |v|) from 0: a NaN never becomes the maximum
        const float m = fabsf(v);
        const float amax = warp_max(m == m ? m : 0.0f);
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const int bi = b & 3;
        const int u = (bi * 32 + lane) >> 4;  // 16-byte unit of the chunk row
        unsigned char* blk = a.act + (static_cast<size_t>(b >> 2) * ncol + ct) * actb;
        blk[c * kTailChunk + ((u ^ (c & 7)) << 4) + (lane & 15)] =
            static_cast<unsigned char>(static_cast<int8_t>(__float2int_rn(__fmul_rn(v, id))));  // NaN -> 0
        if (lane == 0) reinterpret_cast<float*>(blk + a.nt * kTailChunk)[bi * a.nt + c] = d;
      }
    }
  }
}

// ------------------------------------------------------ quantised heads ----
__device__ __forceinline__ void raise_tail(unsigned bits) { atomicOr(&g_tail_status, bits); }

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t& r0, uint32_t& r1, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Global -> this CTA's shared memory without a cache hint (both addresses
// 16-byte aligned, bytes a multiple of 16).  Never multicast.
__device__ __forceinline__ void bulk_g2s_plain(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Bulk prefetch of global memory into L2 (16-byte aligned, bytes a multiple
// of 16); nothing lands in shared memory and nothing waits for it.
__device__ __forceinline__ void prefetch_l2(const void* src_gmem, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src_gmem), "r"(bytes) : "memory");
}
// D = A * B + C over one 32-element block; C = the bits of 1.5 * 2^23, so that
// D, read as a float, is 1.5 * 2^23 + (block sum): |sum| <= 32 * 127 * 128 < 2^22.
__device__ __forceinline__ void mma_block(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(kMagicBits));
}
// Four packed Q4 codes (stored value + 8 in [0, 15]) -> four int8 in [-8, 7].
__device__ __forceinline__ uint32_t q4_codes(uint32_t nib) {
  return ((nib | 0x80808080u) - 0x08080808u) ^ 0x80808080u;
}

template <bool kQ4>
struct TileBytes {
  static constexpr int AB = kQ4 ? kTailChunk / 2 : kTailChunk;  // weight bytes of a row's chunk
  static constexpr int A = kTailRows * AB;
  static constexpr int TB = A + kTailRows * 8;                   // + 4 fp16 scales per row
};

template <int NT, bool kQ4>
struct HeadCfg {
  static constexpr int WN = NT < 32 ? NT : 32;  // token columns of one warp
  static constexpr int WARPS_N = NT / WN;
  static constexpr int WARPS_M = kConsumers / WARPS_N;
  static constexpr int WM = kTailRows / WARPS_M;  // vocab rows of one warp
  static constexpr int MI = WM / 16, NI = WN / 8;
  static constexpr int TB = TileBytes<kQ4>::TB;
  static constexpr int ACTB = NT * (kTailChunk + 16);  // one activation block: codes + [4][NT] scales
  static constexpr int STAGE = TB + ACTB;
  static constexpr int STAGES = (110 * 1024) / STAGE > 6 ? 6 : (110 * 1024) / STAGE;
  static constexpr int DATA = STAGES * STAGE;
  static constexpr int SMEM = DATA + 2 * STAGES * 8 + 16;
};

// Persistent: CTA b takes the work items b, b + G, b + 2G, ... of the
// (head tile, token tile) grid, token tiles fastest, so the CTAs that share a
// weight tile run together and all but the first read it from L2.  Warp 8
// (lane 0) keeps one ring of STAGES shared-memory stages full across all of
// the CTA's items: chunk g goes to stage g % STAGES as one bulk copy of the
// head block and one of the activation block, counted on full[s]; the
// consumer warps release a stage on empty[s].  The kernel runs after the norm
// kernel with programmatic dependent launch: the weights of the first stages
// are requested before griddepcontrol.wait, the activations after it.  Every
// wait is bounded: on a timeout the kernel records kErrTailWait, stops, waits
// (bounded) for the copies it issued and returns.
template <int NT, bool kQ4>
__global__ void __launch_bounds__(kHeadThreads, 2) tail_head_q_kernel(TailHead h, TailArgs a) {
  using C = HeadCfg<NT, kQ4>;
  extern __shared__ __align__(128) unsigned char sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + C::DATA);
  uint64_t* empty = full + C::STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + C::STAGES);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ncol = a.n_pad / NT;
  const int items = h.ntile * ncol;
  const int nkc = h.nkc;
  const int G = gridDim.x;
  grid_release();  // the next kernel may be scheduled; a programmatic one waits for this grid
  if (tid == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    *abort_flag = 0;
  }
  __syncthreads();

  if (warp == kConsumers) {
    if (lane == 0) {
      const int mine = blockIdx.x < items ? (items - blockIdx.x + G - 1) / G : 0;
      const int total = mine * nkc;
      auto stage_of = [&](int g) { return sm + (g % C::STAGES) * C::STAGE; };
      auto issue_head = [&](int g) {
        const int j = g / nkc, kc = g - j * nkc;
        const int tile = (blockIdx.x + j * G) / ncol;
        mbar_expect_tx(&full[g % C::STAGES], C::STAGE);
        bulk_g2s_plain(stage_of(g), h.tiles + (static_cast<size_t>(tile) * nkc + kc) * C::TB, C::TB,
                       &full[g % C::STAGES]);
      };
      auto issue_acts = [&](int g) {
        const int j = g / nkc, kc = g - j * nkc;
        const int ct = (blockIdx.x + j * G) % ncol;
        bulk_g2s_plain(stage_of(g) + C::TB, a.act + (static_cast<size_t>(kc) * ncol + ct) * C::ACTB, C::ACTB,
                       &full[g % C::STAGES]);
      };
      const int pre = total < C::STAGES ? total : C::STAGES;
      for (int g = 0; g < pre; ++g) issue_head(g);
      // While the norm kernel still runs, pull the next head blocks into L2
      // too (no shared memory, no completion to wait for): the stages that
      // follow the wait then read them from L2 and HBM stays busy meanwhile.
      for (int g = pre; g < total && g < pre + kL2Ahead; ++g) {
        const int j = g / nkc, kc = g - j * nkc;
        const int tile = (blockIdx.x + j * G) / ncol;
        prefetch_l2(h.tiles + (static_cast<size_t>(tile) * nkc + kc) * C::TB, C::TB);
      }
      grid_wait();  // the norm kernel's activations are complete and visible
      for (int g = 0; g < pre; ++g) issue_acts(g);
      int issued = pre;
      for (int g = pre; g < total; ++g) {
        if (!mbar_wait_bounded(&empty[g % C::STAGES], ((g / C::STAGES) - 1) & 1)) {
          *abort_flag = 1;
          raise_tail(kErrTailWait);
          break;
        }
        if (*abort_flag) break;
        issue_head(g);
        issue_acts(g);
        ++issued;
      }
      // no copy may still be in flight when the CTA's shared memory goes away
      for (int g = issued > C::STAGES ? issued - C::STAGES : 0; g < issued; ++g)
        (void)mbar_wait_bounded(&full[g % C::STAGES], (g / C::STAGES) & 1);
    }
    return;
  }

  const int wm = warp % C::WARPS_M, wn = warp / C::WARPS_M;
  int g = 0;
  for (int it = blockIdx.x; it < items; it += G) {
    const int tile = it / ncol, col0 = (it % ncol) * NT;
    float2 acc[C::MI][C::NI][2];  // [..][..][0]: row g, tokens 2t, 2t+1; [1]: row g + 8
#pragma unroll
    for (int mi = 0; mi < C::MI; ++mi)
#pragma unroll
      for (int ni = 0; ni < C::NI; ++ni) acc[mi][ni][0] = acc[mi][ni][1] = make_float2(0.0f, 0.0f);
    for (int kc = 0; kc < nkc; ++kc, ++g) {
      const int s = g % C::STAGES;
      if (!mbar_wait_bounded(&full[s], (g / C::STAGES) & 1)) {
        *abort_flag = 1;
        raise_tail(kErrTailWait);
        return;
      }
      const unsigned char* A = sm + s * C::STAGE;
      const unsigned char* WS = A + TileBytes<kQ4>::A;
      const unsigned char* B = A + C::TB;
      const float* XS = reinterpret_cast<const float*>(B + NT * kTailChunk);
      uint2 wraw[C::MI][2];  // 4 fp16 scales of each of my rows
#pragma unroll
      for (int mi = 0; mi < C::MI; ++mi)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
          wraw[mi][hh] = *reinterpret_cast<const uint2*>(WS + (wm * C::WM + mi * 16 + (lane >> 2) + hh * 8) * 8);

#pragma unroll
      for (int bi = 0; bi < 4; ++bi) {
        uint32_t af[C::MI][4];
#pragma unroll
        for (int mi = 0; mi < C::MI; ++mi) {
          if constexpr (!kQ4) {
            const int m = lane >> 3;
            const int r = wm * C::WM + mi * 16 + ((m & 1) << 3) + (lane & 7);
            const int u = 2 * bi + (m >> 1);
            ldsm_x4(af[mi][0], af[mi][1], af[mi][2], af[mi][3], A + r * 128 + ((u ^ (r & 7)) << 4));
          } else {
            const int r = wm * C::WM + mi * 16 + (lane >> 2);
            const int r8 = r + 8;
            const uint32_t p0 =
                *reinterpret_cast<const uint32_t*>(A + r * 64 + ((bi ^ ((r >> 1) & 3)) << 4) + 4 * (lane & 3));
            const uint32_t p1 =
                *reinterpret_cast<const uint32_t*>(A + r8 * 64 + ((bi ^ ((r8 >> 1) & 3)) << 4) + 4 * (lane & 3));
            af[mi][0] = q4_codes(p0 & 0x0F0F0F0Fu);
            af[mi][1] = q4_codes(p1 & 0x0F0F0F0Fu);
            af[mi][2] = q4_codes((p0 >> 4) & 0x0F0F0F0Fu);
            af[mi][3] = q4_codes((p1 >> 4) & 0x0F0F0F0Fu);
          }
        }
        uint32_t bf[C::NI][2];
        if constexpr (C::NI == 1) {
          const int m = (lane >> 3) & 1;
          const int c = wn * C::WN + (lane & 7);
          const int u = 2 * bi + m;
          ldsm_x2(bf[0][0], bf[0][1], B + c * kTailChunk + ((u ^ (c & 7)) << 4));
        } else {
#pragma unroll
          for (int ni = 0; ni < C::NI; ni += 2) {
            const int m = lane >> 3;
            const int c = wn * C::WN + (ni + (m >> 1)) * 8 + (lane & 7);
            const int u = 2 * bi + (m & 1);
            ldsm_x4(bf[ni][0], bf[ni][1], bf[ni + 1][0], bf[ni + 1][1], B + c * kTailChunk + ((u ^ (c & 7)) << 4));
          }
        }
#pragma unroll
        for (int mi = 0; mi < C::MI; ++mi) {
          float w[2];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const uint32_t word = bi < 2 ? wraw[mi][hh].x : wraw[mi][hh].y;
            w[hh] = __half2float(__ushort_as_half(static_cast<unsigned short>(bi & 1 ? word >> 16 : word)));
          }
#pragma unroll
          for (int ni = 0; ni < C::NI; ++ni) {
            int d[4];
            mma_block(d, af[mi], bf[ni][0], bf[ni][1]);
            const float2 xs2 = *reinterpret_cast<const float2*>(XS + bi * NT + wn * C::WN + ni * 8 + 2 * (lane & 3));
            const float2 neg = make_float2(-kMagic, -kMagic);
            const float2 f01 = __fadd2_rn(make_float2(__int_as_float(d[0]), __int_as_float(d[1])), neg);
            const float2 f23 = __fadd2_rn(make_float2(__int_as_float(d[2]), __int_as_float(d[3])), neg);
            const float2 c01 = __fmul2_rn(make_float2(w[0], w[0]), xs2);
            const float2 c23 = __fmul2_rn(make_float2(w[1], w[1]), xs2);
            acc[mi][ni][0] = __ffma2_rn(c01, f01, acc[mi][ni][0]);
            acc[mi][ni][1] = __ffma2_rn(c23, f23, acc[mi][ni][1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // straight from registers: for each token a warp writes 8 consecutive
    // logits (one 32-byte sector) per row group
    const int row0 = tile * kTailRows + wm * C::WM + (lane >> 2);
    const int c0 = col0 + wn * C::WN + 2 * (lane & 3);
#pragma unroll
    for (int mi = 0; mi < C::MI; ++mi)
#pragma unroll
      for (int ni = 0; ni < C::NI; ++ni)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int r = row0 + mi * 16 + hh * 8;
          const int c = c0 + ni * 8;
          if (r < h.vocab) {
            if (c < a.n) a.logits[static_cast<long long>(c) * a.ld + r] = acc[mi][ni][hh].x;
            if (c + 1 < a.n) a.logits[static_cast<long long>(c + 1) * a.ld + r] = acc[mi][ni][hh].y;
          }
        }
  }
}

// ------------------------------------------------------------ F32 head ----
// The same persistent ring as the quantised heads, for an fp32 head packed
// tile-major (kTailRows rows x kF32K floats per 16 KB block, 16-byte units
// XOR-swizzled by (row & 7)): a producer warp streams each block and the
// matching activation block ([kF32K][NT] floats from the norm kernel) with
// bulk copies; four consumer warps hold one vocab row per thread and NT
// tokens, and add the products in index order, each rounded, as the
// reference's dot_f32.  Scalar __fmul_rn / __fadd_rn: the packed float2 forms
// are fused into one FFMA2 by the compiler, which the reference's separate
// roundings forbid.
constexpr int kF32K = 32;                                  // K floats per block
constexpr int kF32Block = kTailRows * kF32K * 4;           // 16 KB
constexpr int kF32Consumers = kTailRows / 32;              // one row per consumer thread
constexpr int kF32Threads = (kF32Consumers + 1) * 32;

template <int NT>
struct F32Cfg {
  static constexpr int XB = kF32K * NT * 4;  // one activation block
  static constexpr int STAGE = kF32Block + XB;
  static constexpr int STAGES = (110 * 1024) / STAGE > 6 ? 6 : (110 * 1024) / STAGE;
  static constexpr int DATA = STAGES * STAGE;
  static constexpr int SMEM = DATA + 2 * STAGES * 8 + 16;
};

template <int NT>
__global__ void __launch_bounds__(kF32Threads, 2) tail_head_f32_kernel(TailHead h, TailArgs a) {
  using C = F32Cfg<NT>;
  extern __shared__ __align__(128) unsigned char sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + C::DATA);
  uint64_t* empty = full + C::STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + C::STAGES);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ncol = a.n_pad / NT;
  const int items = h.ntile * ncol;
  const int nk = h.dim / kF32K;
  const int G = gridDim.x;
  grid_release();  // the next kernel may be scheduled; a programmatic one waits for this grid
  if (tid == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kF32Consumers);
    }
    *abort_flag = 0;
  }
  __syncthreads();

  if (warp == kF32Consumers) {
    if (lane == 0) {
      const int mine = blockIdx.x < items ? (items - blockIdx.x + G - 1) / G : 0;
      const int total = mine * nk;
      auto stage_of = [&](int g) { return sm + (g % C::STAGES) * C::STAGE; };
      auto block_of = [&](int g) {
        const int j = g / nk, kc = g - j * nk;
        const int tile = (blockIdx.x + j * G) / ncol;
        return h.tiles + (static_cast<size_t>(tile) * nk + kc) * kF32Block;
      };
      auto issue_head = [&](int g) {
        mbar_expect_tx(&full[g % C::STAGES], C::STAGE);
        bulk_g2s_plain(stage_of(g), block_of(g), kF32Block, &full[g % C::STAGES]);
      };
      auto issue_acts = [&](int g) {
        const int j = g / nk, kc = g - j * nk;
        const int ct = (blockIdx.x + j * G) % ncol;
        bulk_g2s_plain(stage_of(g) + kF32Block,
                       reinterpret_cast<const unsigned char*>(a.xb) + (static_cast<size_t>(kc) * ncol + ct) * C::XB,
                       C::XB, &full[g % C::STAGES]);
      };
      const int pre = total < C::STAGES ? total : C::STAGES;
      for (int g = 0; g < pre; ++g) issue_head(g);
      for (int g = pre; g < total && g < pre + kL2Ahead; ++g) prefetch_l2(block_of(g), kF32Block);
      grid_wait();  // the norm kernel's activations are complete and visible
      for (int g = 0; g < pre; ++g) issue_acts(g);
      int issued = pre;
      for (int g = pre; g < total; ++g) {
        if (!mbar_wait_bounded(&empty[g % C::STAGES], ((g / C::STAGES) - 1) & 1)) {
          *abort_flag = 1;
          raise_tail(kErrTailWait);
          break;
        }
        if (*abort_flag) break;
        issue_head(g);
        issue_acts(g);
        ++issued;
      }
      // no copy may still be in flight when the CTA's shared memory goes away
      for (int g = issued > C::STAGES ? issued - C::STAGES : 0; g < issued; ++g)
        (void)mbar_wait_bounded(&full[g % C::STAGES], (g / C::STAGES) & 1);
    }
    return;
  }

  const int r = tid;  // this thread's row of the tile
  int g = 0;
  for (int it = blockIdx.x; it < items; it += G) {
    const int tile = it / ncol, col0 = (it % ncol) * NT;
    float2 acc[NT / 2];
#pragma unroll
    for (int j = 0; j < NT / 2; ++j) acc[j] = make_float2(0.0f, 0.0f);
    for (int kc = 0; kc < nk; ++kc, ++g) {
      const int s = g % C::STAGES;
      if (!mbar_wait_bounded(&full[s], (g / C::STAGES) & 1)) {
        *abort_flag = 1;
        raise_tail(kErrTailWait);
        return;
      }
      const unsigned char* W = sm + s * C::STAGE;
      const float* X = reinterpret_cast<const float*>(W + kF32Block);  // [kF32K][NT]
#pragma unroll
      for (int u = 0; u < kF32K / 4; ++u) {
        const float4 wv = *reinterpret_cast<const float4*>(W + r * (kF32K * 4) + ((u ^ (r & 7)) << 4));
        const float we[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
#pragma unroll
          for (int j = 0; j < NT / 2; ++j) {
            const float2 xv = *reinterpret_cast<const float2*>(X + (4 * u + e) * NT + 2 * j);
            acc[j].x = __fadd_rn(acc[j].x, __fmul_rn(we[e], xv.x));
            acc[j].y = __fadd_rn(acc[j].y, __fmul_rn(we[e], xv.y));
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    const int row = tile * kTailRows + r;
    if (row < h.vocab) {
#pragma unroll
      for (int j = 0; j < NT / 2; ++j) {
        if (col0 + 2 * j < a.n) a.logits[static_cast<long long>(col0 + 2 * j) * a.ld + row] = acc[j].x;
        if (col0 + 2 * j + 1 < a.n) a.logits[static_cast<long long>(col0 + 2 * j + 1) * a.ld + row] = acc[j].y;
      }
    }
  }
}

template <int NT, bool kQ4>
cudaError_t launch_head_q(const TailHead& h, const TailArgs& a, cudaStream_t s) {
  using C = HeadCfg<NT, kQ4>;
  auto kern = tail_head_q_kernel<NT, kQ4>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  // the fewest items per CTA that two CTAs per SM allow, then the fewest CTAs
  // that carry them: every CTA ends up with the same count, give or take one
  const int items = h.ntile * (a.n_pad / NT);
  const int per = (items + 2 * sms - 1) / (2 * sms);
  const int grid = (items + per - 1) / per;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kHeadThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, h, a);
}

template <bool kQ4>
cudaError_t launch_head_q_nt(const TailHead& h, const TailArgs& a, cudaStream_t s) {
  switch (a.nt) {
    case 8:
      return launch_head_q<8, kQ4>(h, a, s);
    case 16:
      return launch_head_q<16, kQ4>(h, a, s);
    case 32:
      return launch_head_q<32, kQ4>(h, a, s);
    default:
      return launch_head_q<64, kQ4>(h, a, s);
  }
}

template <int NT>
cudaError_t launch_head_f32(const TailHead& h, const TailArgs& a, cudaStream_t s) {
  using C = F32Cfg<NT>;
  auto kern = tail_head_f32_kernel<NT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  const int items = h.ntile * (a.n_pad / NT);
  const int per = (items + 2 * sms - 1) / (2 * sms);
  const int grid = (items + per - 1) / per;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kF32Threads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, h, a);
}

// ---------------------------------------------- Q8 heads, > 32 tokens ----
// tcgen05 form of the quantised head for batches: one CTA per SM, persistent
// over work items (head tile of M = 128 vocab rows, token tile of N = 64 or
// 128 tokens), token tiles fastest, so that the CTAs sharing a head tile run
// together and all but one read it from L2.  The operands stay in the
// layouts the mma.sync kernel streams: a head block is 128 rows x 128 bytes
// of K with 16-byte units XOR-swizzled by (row & 7), an activation block N
// token rows the same way, which is the tensor cores' K-major 128-byte-swizzle
// layout.
//
//   warp 0 (lane 0)   streams each chunk of 4 K blocks (the activation codes
//                     and the head block with its fp16 scales) into a ring of
//                     shared-memory stages with bulk copies (full / empty);
//   warp 1 (lane 0)   issues one tcgen05.mma kind::i8 per 32-element block,
//                     D = A_b * B_b^T + D, into the next of 512 / N
//                     accumulators in tensor memory, and commits it to that
//                     accumulator's barrier;
//   warps 2..17       the epilogue: warp w reads tensor-memory lanes
//                     32 (w mod 4) .. +31 (its vocab rows) and a quarter of
//                     the token columns of one block, refills the accumulator
//                     with the bits of 1.5 * 2^23 (so that the next block's D,
//                     read as a float, is 1.5 * 2^23 + its block sum, exact
//                     since |sum| < 2^22) and releases it, then applies the
//                     reference's r = fma(sw * sx, float(sum), r) in block order.
//
// Every wait is bounded; a timeout records kErrTailWait and the CTA stops.
constexpr int kTcEpiWarps = 16;
constexpr int kTcThreads = (2 + kTcEpiWarps) * 32;
constexpr int kTcStages = 4;
constexpr size_t kTcSmemLimit = 227 * 1024;

template <int N>
struct TcCfg {
  static constexpr int CTAS = N == 64 ? 2 : 1;                  // resident CTAs per SM
  static constexpr int STAGES = N == 64 ? 3 : kTcStages;
  static constexpr int ACT = N * kTailChunk;                    // one chunk's activation codes
  static constexpr int HEAD = TileBytes<false>::TB;             // a head block: weights + scales
  static constexpr int STAGE = ACT + ((HEAD + 1023) & ~1023);   // parts 1024-byte aligned
  static constexpr int CPT = N / 4;                             // token columns per epilogue thread
  static constexpr uint32_t COLS = 512 / CTAS;                  // this CTA's share of tensor memory
  static constexpr int NBUF = COLS / N;                         // accumulators
  static size_t smem(int nkc) {
    return 1024 + static_cast<size_t>(STAGES) * STAGE + static_cast<size_t>(nkc) * 4 * N * 4 + 64 * NBUF + 256;
  }
};

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (start address in 16-byte units, SM100 descriptor version 1).
__device__ __forceinline__ uint64_t tc_desc(const void* p) {
  const uint64_t addr = (smem_u32(p) >> 4) & 0x3FFFu;
  return addr | (1ull << 16) | (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// D[tmem] = A * B^T (+ D when accumulate), 128 x N, int8 x int8 -> int32.
__device__ __forceinline__ void tc_mma_i8(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// 8 consecutive 32-bit columns of this warp's 32 lanes; complete after tc_wait_ld.
__device__ __forceinline__ void tc_ld8_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 4 consecutive floats of shared memory, in program order (not hoisted).
__device__ __forceinline__ float4 lds4(const float* p) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(smem_u32(p)));
  return v;
}
// The magic bits into 16 consecutive columns of this warp's 32 lanes.
constexpr uint32_t kMagicU = static_cast<uint32_t>(kMagicBits);
__device__ __forceinline__ void tc_st16_magic(uint32_t taddr) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(kMagicU), "r"(kMagicU), "r"(kMagicU), "r"(kMagicU), "r"(kMagicU), "r"(kMagicU), "r"(kMagicU), "r"(kMagicU),
      "r"(kMagicU), "r"(kMagicU), "r"(kMagicU), "r"(kMagicU), "r"(kMagicU), "r"(kMagicU), "r"(kMagicU), "r"(kMagicU)
      : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <int N>
__global__ void __launch_bounds__(kTcThreads, TcCfg<N>::CTAS) tail_head_tc_kernel(TailHead h, TailArgs a) {
  using C = TcCfg<N>;
  extern __shared__ __align__(1024) unsigned char sm_raw[];
  // the 128-byte swizzle is a function of the address: stages start 1024-aligned
  unsigned char* sm = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);
  const int nkc = h.nkc, nb = h.dim / kTailBlk;
  const int ncol = a.n_pad / N;
  const int items = h.ntile * ncol;
  const int G = gridDim.x;            // a multiple of ncol: this CTA's token tile never changes
  const int ct = static_cast<int>(blockIdx.x) % ncol;
  float* XS = reinterpret_cast<float*>(sm + C::STAGES * C::STAGE);  // [nkc][4][N] scales of token tile ct
  uint64_t* full = reinterpret_cast<uint64_t*>(XS + static_cast<size_t>(nkc) * 4 * N);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accf = empty + C::STAGES;  // [NBUF] an accumulator holds a finished block
  uint64_t* acce = accf + C::NBUF;     // [NBUF] an accumulator was read and refilled
  uint32_t* tslot = reinterpret_cast<uint32_t*>(acce + C::NBUF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t actb = static_cast<size_t>(N) * (kTailChunk + 16);
  grid_release();  // the next kernel may be scheduled; a programmatic one waits for this grid
  if (tid == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + kTcEpiWarps);  // the MMAs' commit + every epilogue warp (head scales read)
    }
    for (int i = 0; i < C::NBUF; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], kTcEpiWarps);
    }
    *abort_flag = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(C::COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  grid_wait();  // the norm kernel's activation blocks are complete and visible
  for (int i = tid; i < nkc * 4 * N; i += kTcThreads) {
    const int kc = i / (4 * N);
    XS[i] = reinterpret_cast<const float*>(a.act + (static_cast<size_t>(kc) * ncol + ct) * actb +
                                           N * kTailChunk)[i - kc * 4 * N];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const int q = warp & 3, grp = (warp - 2) >> 2;  // epilogue: lane quadrant, token quarter
  const uint32_t tl = tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(grp * C::CPT);

  const int mine = static_cast<int>(blockIdx.x) < items ? (items - static_cast<int>(blockIdx.x) + G - 1) / G : 0;
  const int total = mine * nkc;  // chunks this CTA streams
  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int g = 0; g < total; ++g) {
        const int s = g % C::STAGES;
        if (g >= C::STAGES && !mbar_wait_bounded(&empty[s], ((g / C::STAGES) - 1) & 1)) {
          *abort_flag = 1;
          raise_tail(kErrTailWait);
          break;
        }
        if (*abort_flag) break;
        const int j = g / nkc, kc = g - j * nkc;
        const int tile = (static_cast<int>(blockIdx.x) + j * G) / ncol;
        unsigned char* st = sm + s * C::STAGE;
        mbar_expect_tx(&full[s], C::ACT + C::HEAD);
        bulk_g2s_plain(st, a.act + (static_cast<size_t>(kc) * ncol + ct) * actb, C::ACT, &full[s]);
        bulk_g2s_plain(st + C::ACT, h.tiles + (static_cast<size_t>(tile) * nkc + kc) * C::HEAD, C::HEAD, &full[s]);
        ++issued;
      }
      // no copy may still be in flight when the CTA's shared memory goes away
      for (int g = issued > C::STAGES ? issued - C::STAGES : 0; g < issued; ++g)
        (void)mbar_wait_bounded(&full[g % C::STAGES], (g / C::STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // kind::i8: D s32, A and B signed int8, both K-major, N >> 3 at bit 17, M (128) >> 4 at bit 24
      const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) | (8u << 24);
      int gb = 0;
      for (int g = 0; g < total && !*abort_flag; ++g) {
        const int s = g % C::STAGES;
        if (!mbar_wait_bounded(&full[s], (g / C::STAGES) & 1)) {
          *abort_flag = 1;
          raise_tail(kErrTailWait);
          break;
        }
        tc_fence_after();
        const unsigned char* st = sm + s * C::STAGE;
        bool ok = true;
        for (int bi = 0; bi < 4; ++bi, ++gb) {
          const int ab = gb % C::NBUF;
          if (!mbar_wait_bounded(&acce[ab], ((gb / C::NBUF) & 1) ^ 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          tc_mma_i8(tmem + static_cast<uint32_t>(ab * N), tc_desc(st + C::ACT + 32 * bi), tc_desc(st + 32 * bi), idesc,
                    0u);  // D = the block's sums alone
          tc_commit(&accf[ab]);
        }
        if (!ok) {
          *abort_flag = 1;
          raise_tail(kErrTailWait);
          break;
        }
        tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
      }
    }
  } else {
    const float2 neg = make_float2(-kMagic, -kMagic);
    const int row = 32 * q + lane;  // vocab row within the tile
    int g = 0, gb = 0;
    for (int j = 0; j < mine && !*abort_flag; ++j) {
      const int tile = (static_cast<int>(blockIdx.x) + j * G) / ncol;
      float2 acc[C::CPT / 2];
#pragma unroll
      for (int i = 0; i < C::CPT / 2; ++i) acc[i] = make_float2(0.0f, 0.0f);
      bool ok = true;
      for (int kc = 0; kc < nkc && ok; ++kc, ++g) {
        const int s = g % C::STAGES;
        if (!mbar_wait_bounded(&full[s], (g / C::STAGES) & 1)) {
          ok = false;
          break;
        }
        // this row's four fp16 block scales of the chunk, then the stage may go
        const uint2 wr = *reinterpret_cast<const uint2*>(sm + s * C::STAGE + C::ACT + TileBytes<false>::A + row * 8);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll 1
        for (int bi = 0; bi < 4; ++bi, ++gb) {
          const int ab = gb % C::NBUF;
          if (!mbar_wait_bounded(&accf[ab], (gb / C::NBUF) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // the block's sums out of tensor memory, the accumulator released at once
          uint32_t d[C::CPT];
#pragma unroll
          for (int c = 0; c < C::CPT; c += 8) tc_ld8_nowait(tl + static_cast<uint32_t>(ab * N + c), d + c);
          tc_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce[ab]);
          if (kc * 4 + bi < nb) {  // blocks past dim (zero padding) are not in the reference's sum
            const uint32_t wword = bi < 2 ? wr.x : wr.y;
            const float wf = __half2float(__ushort_as_half(static_cast<unsigned short>(bi & 1 ? wword >> 16 : wword)));
            const float2 ww = make_float2(wf, wf);
            const float* xs = XS + (kc * 4 + bi) * N + grp * C::CPT;
#pragma unroll
            for (int e = 0; e < C::CPT; e += 4) {
              const float4 x4 = lds4(xs + e);
              const float2 c01 = __fmul2_rn(ww, make_float2(x4.x, x4.y));
              const float2 c23 = __fmul2_rn(ww, make_float2(x4.z, x4.w));
              // float(sum) exactly: the bits of 1.5 * 2^23 + sum (|sum| < 2^22), less 1.5 * 2^23
              const float2 f01 = __fadd2_rn(
                  make_float2(__uint_as_float(d[e] + kMagicU), __uint_as_float(d[e + 1] + kMagicU)), neg);
              const float2 f23 = __fadd2_rn(
                  make_float2(__uint_as_float(d[e + 2] + kMagicU), __uint_as_float(d[e + 3] + kMagicU)), neg);
              acc[e / 2] = __ffma2_rn(c01, f01, acc[e / 2]);
              acc[e / 2 + 1] = __ffma2_rn(c23, f23, acc[e / 2 + 1]);
            }
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        raise_tail(kErrTailWait);
        break;
      }
      const int v = tile * kTailRows + row;
      if (v < h.vocab) {
#pragma unroll
        for (int c = 0; c < C::CPT; c += 2) {
          const int t = ct * N + grp * C::CPT + c;
          if (t < a.n) a.logits[static_cast<long long>(t) * a.ld + v] = acc[c / 2].x;
          if (t + 1 < a.n) a.logits[static_cast<long long>(t + 1) * a.ld + v] = acc[c / 2].y;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::COLS) : "memory");
}

template <int N>
cudaError_t launch_head_tc(const TailHead& h, const TailArgs& a, cudaStream_t s) {
  using C = TcCfg<N>;
  auto kern = tail_head_tc_kernel<N>;
  const size_t smem = C::smem(h.nkc);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  // persistent, one CTA per SM, a multiple of the token tiles so that each
  // CTA keeps one token tile; the fewest items per CTA, then the fewest CTAs
  const int ncol = a.n_pad / N, items = h.ntile * ncol;
  const int slots = C::CTAS * sms / ncol * ncol;
  const int per = (items + slots - 1) / slots;
  const int grid = (items + per * ncol - 1) / (per * ncol) * ncol;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, h, a);
}

// Token tile of the tcgen05 path (0: the mma.sync path): Q8 heads, more than
// 32 tokens, when the stages and the resident activation scales fit, and only
// when VERBO_CUDA_TAIL_TCGEN05=1 selects it: measured on B200 it is slower
// than the mma.sync kernel (each epilogue warp waits out the tensor-memory
// load of every block before it can use it), so it is not the default.
int tc_tokens(const TailHead& h, int n) {
  const char* sel = std::getenv("VERBO_CUDA_TAIL_TCGEN05");
  if (!sel || sel[0] != '1' || sel[1] != '\0') return 0;
  if (h.dtype != kTailQ8 || n <= 32) return 0;
  const int N = 64;
  if ((n + N - 1) / N > 16) return 0;  // at most 16 token tiles (the grid holds a multiple of them)
  const size_t need = N == 64 ? TcCfg<64>::smem(h.nkc) : TcCfg<128>::smem(h.nkc);
  return need <= kTcSmemLimit ? N : 0;
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

}  // namespace

size_t tail_tiles_bytes(int dtype, int vocab, int dim) {
  const size_t ntile = (vocab + kTailRows - 1) / kTailRows;
  if (dtype == kTailF32) return ntile * (dim / kF32K) * kF32Block;
  const size_t nkc = (dim + kTailChunk - 1) / kTailChunk;
  return ntile * nkc * (dtype == kTailQ4 ? TileBytes<true>::TB : TileBytes<false>::TB);
}

void tail_pack_tiles(int dtype, int vocab, int dim, const void* q, const uint16_t* s, unsigned char* out) {
  if (dtype == kTailF32) {  // blocks of kTailRows rows x kF32K floats, 16-byte units swizzled by (row & 7)
    const int ntile = (vocab + kTailRows - 1) / kTailRows, nk = dim / kF32K;
    std::memset(out, 0, tail_tiles_bytes(dtype, vocab, dim));
    const unsigned char* src = static_cast<const unsigned char*>(q);
    for (int t = 0; t < ntile; ++t)
      for (int kc = 0; kc < nk; ++kc) {
        unsigned char* blk = out + (static_cast<size_t>(t) * nk + kc) * kF32Block;
        for (int r = 0; r < kTailRows && t * kTailRows + r < vocab; ++r) {
          const unsigned char* row = src + (static_cast<size_t>(t) * kTailRows + r) * dim * 4 + kc * kF32K * 4;
          for (int u = 0; u < kF32K / 4; ++u) std::memcpy(blk + r * kF32K * 4 + ((u ^ (r & 7)) << 4), row + u * 16, 16);
        }
      }
    return;
  }
  const bool q4 = dtype == kTailQ4;
  const int ab = q4 ? TileBytes<true>::AB : TileBytes<false>::AB;
  const size_t tb = q4 ? TileBytes<true>::TB : TileBytes<false>::TB;
  const int rowbytes = q4 ? dim / 2 : dim, nb = dim / kTailBlk;
  const int ntile = (vocab + kTailRows - 1) / kTailRows, nkc = (dim + kTailChunk - 1) / kTailChunk;
  std::memset(out, 0, tail_tiles_bytes(dtype, vocab, dim));
  const unsigned char* src = static_cast<const unsigned char*>(q);
  for (int t = 0; t < ntile; ++t)
    for (int kc = 0; kc < nkc; ++kc) {
      unsigned char* blk = out + (static_cast<size_t>(t) * nkc + kc) * tb;
      for (int r = 0; r < kTailRows && t * kTailRows + r < vocab; ++r) {
        const size_t gr = static_cast<size_t>(t) * kTailRows + r;
        for (int u = 0; u < ab / 16; ++u) {
          const int off = kc * ab + u * 16;
          if (off >= rowbytes) break;
          const int su = q4 ? (u ^ ((r >> 1) & 3)) : (u ^ (r & 7));
          std::memcpy(blk + r * ab + su * 16, src + gr * rowbytes + off, 16);
        }
        for (int j = 0; j < 4 && kc * 4 + j < nb; ++j)
          std::memcpy(blk + kTailRows * ab + r * 8 + j * 2, s + gr * nb + kc * 4 + j, 2);
      }
    }
}

int tail_token_tile(const TailHead& h, int n) {
  if (h.dtype == kTailF32) return n <= 2 ? 2 : n <= 4 ? 4 : n <= 8 ? 8 : 16;
  if (const int N = tc_tokens(h, n)) return N;  // every token in one tensor-core tile
  return n <= 8 ? 8 : n <= 16 ? 16 : n <= 32 ? 32 : 64;
}

size_t tail_scratch_bytes(const TailHead& h, int n) {
  const int nt = tail_token_tile(h, n);
  const size_t n_pad = static_cast<size_t>((n + nt - 1) / nt) * nt;
  if (h.dtype == kTailF32) return align256(static_cast<size_t>(h.dim) * n_pad * 4);
  return align256(static_cast<size_t>(h.nkc) * n_pad * (kTailChunk + 16));
}

void tail_scratch_attach(const TailHead& h, int n, void* base, TailArgs& a) {
  a.nt = tail_token_tile(h, n);
  a.n_pad = (n + a.nt - 1) / a.nt * a.nt;
  a.act = nullptr;
  a.xb = nullptr;
  if (h.dtype == kTailF32)
    a.xb = static_cast<float*>(base);
  else
    a.act = static_cast<unsigned char*>(base);
}

cudaError_t launch_tail(const TailHead& h, const TailArgs& a, cudaStream_t s) {
  if (a.n <= 0) return cudaSuccess;
  const int norm_smem = h.dim * 8;
  cudaError_t e = cudaFuncSetAttribute(tail_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, norm_smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n_pad);
  cfg.blockDim = dim3(kTailThreads);
  cfg.dynamicSmemBytes = norm_smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, tail_norm_kernel, h, a);
  if (e != cudaSuccess) return e;
  switch (h.dtype) {
    case kTailQ8:
      switch (tc_tokens(h, a.n)) {
        case 64:
          return launch_head_tc<64>(h, a, s);
        default:
          return launch_head_q_nt<false>(h, a, s);
      }
    case kTailQ4:
      return launch_head_q_nt<true>(h, a, s);
    default:
      switch (a.nt) {
        case 2:
          return launch_head_f32<2>(h, a, s);
        case 4:
          return launch_head_f32<4>(h, a, s);
        case 8:
          return launch_head_f32<8>(h, a, s);
        default:
          return launch_head_f32<16>(h, a, s);
      }
  }
}

cudaError_t tail_read_status(unsigned* st, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(st, g_tail_status, sizeof(unsigned));
  if (e != cudaSuccess || !clear || !*st) return e;
  const unsigned z = 0;
  return cudaMemcpyToSymbol(g_tail_status, &z, sizeof(unsigned));
}

}  // namespace vb
