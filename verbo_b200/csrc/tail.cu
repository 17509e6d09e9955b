// Kernels of the logits producer tail (src/session.cpp:163-169).
//
// tail_norm_kernel      one warp per hidden row: rmsnorm (src/session.cpp:14-19)
//                       and, for quantised heads, quant_act (src/kernels.cpp:106);
// tail_head_q_kernel    Q8 / Q4 heads: int8 tensor-core MMA, one m16n8k32 per
//                       32-element block, the block's fp32 scale applied in
//                       the epilogue of that MMA (dot_q8 / dot_q4,
//                       src/kernels.cpp:576-600);
// tail_head_f32_kernel  F32 heads: one vocab row per thread (dot_f32,
//                       src/kernels.cpp:570-574).
//
// Every rounding step is the reference scalar build's, in its order: the sum
// of squares runs sequentially, products and sums are rounded separately
// where the reference rounds them separately (__fmul_rn / __fadd_rn are never
// contracted), and the block accumulate is the one FMA the reference's build
// forms, r = fma(scale_w * scale_x, float(block sum), r), in block order.
#include <cuda_fp16.h>

#include "device.cuh"
#include "tail.cuh"

namespace vb {
namespace {

constexpr int kNormChunk = 1024;            // floats of a row staged per warp at a time
constexpr int kMagicBits = 0x4B400000;      // bits of 1.5 * 2^23
constexpr float kMagic = 12582912.0f;       // 1.5 * 2^23
constexpr int kF32Chunk = 512;              // K floats of the F32 kernel's activation stage

// ---------------------------------------------------------------- norm ----
// Lane 0 sums the squares in index order from a staged chunk of the row (the
// reference's loop); the whole warp then normalises, quantises one 32-block
// per step and writes the zero padding up to dimp.
__global__ void __launch_bounds__(kTailThreads) tail_norm_kernel(TailHead h, TailArgs a) {
  __shared__ __align__(16) float stage[kTailThreads / 32][kNormChunk];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * (kTailThreads / 32) + warp;
  if (row >= a.n) return;
  const float* x = a.x + static_cast<long long>(row) * a.ldx;
  float* st = stage[warp];
  float ss = 0.0f;
  for (int c0 = 0; c0 < h.dim; c0 += kNormChunk) {
    const int len = min(kNormChunk, h.dim - c0);  // a multiple of 32
    for (int i = lane; i < len; i += 32) st[i] = x[c0 + i];
    __syncwarp();
    if (lane == 0) {
      for (int i = 0; i < len; i += 4) {
        const float4 v = *reinterpret_cast<const float4*>(st + i);
        ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
        ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
        ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
        ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
      }
    }
    __syncwarp();
  }
  ss = __shfl_sync(0xffffffffu, ss, 0);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(h.dim)), h.eps)));
  const long long qrow = static_cast<long long>(row) * h.dimp;
  for (int b = 0; b < h.nbp; ++b) {
    const int i = b * kTailBlk + lane;
    const float v = i < h.dim ? __fmul_rn(h.norm[i], __fmul_rn(x[i], r)) : 0.0f;
    if (h.dtype == kTailF32) {
      a.xb[qrow + i] = v;
      continue;
    }
    // std::max(amax, |v|) from 0: a NaN never becomes the maximum
    const float m = fabsf(v);
    const float amax = warp_max(m == m ? m : 0.0f);
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    a.xq[qrow + i] = static_cast<int8_t>(__float2int_rn(__fmul_rn(v, id)));  // NaN -> 0
    if (lane == 0) a.xs[static_cast<long long>(row) * h.nbp + b] = d;
  }
}

// ------------------------------------------------------ quantised heads ----
__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(ok ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async8_zfill(void* dst, const void* src, bool ok) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(ok ? 8 : 0)
               : "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t& r0, uint32_t& r1, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
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

template <int NT, bool kQ4>
struct HeadCfg {
  static constexpr int WN = NT < 32 ? NT : 32;         // token columns of one warp
  static constexpr int WARPS_N = NT / WN;
  static constexpr int WARPS_M = (kTailThreads / 32) / WARPS_N;
  static constexpr int WM = kTailRows / WARPS_M;        // vocab rows of one warp
  static constexpr int MI = WM / 16, NI = WN / 8;
  static constexpr int AU = kQ4 ? 4 : 8;                // 16-byte units of a row's chunk
  static constexpr int A_BYTES = kTailRows * AU * 16;
  static constexpr int B_BYTES = NT * kTailChunk;
  static constexpr int WS_BYTES = kTailRows * 8;        // 4 fp16 scales per row
  static constexpr int XS_BYTES = NT * 16;              // 4 fp32 scales per token
  static constexpr int STAGE = A_BYTES + B_BYTES + WS_BYTES + XS_BYTES;
  static constexpr int OUT_LD = kTailRows + 4;
  static constexpr int SMEM = (kTailStages * STAGE > NT * OUT_LD * 4) ? kTailStages * STAGE : NT * OUT_LD * 4;
};

// One CTA: kTailRows vocab rows x NT tokens.  A K-chunk of 4 blocks per
// pipeline stage (cp.async, zero-filled past the vocab, the tokens and dim).
// Shared layouts use an XOR swizzle of the 16-byte units so that ldmatrix and
// the Q4 word loads are conflict-free.  The blockIdx.x (token tiles) runs
// fastest, so the CTAs that share a weight tile run together and read it from
// L2 after the first.
template <int NT, bool kQ4>
__global__ void __launch_bounds__(kTailThreads, 2) tail_head_q_kernel(TailHead h, TailArgs a) {
  using C = HeadCfg<NT, kQ4>;
  extern __shared__ __align__(128) unsigned char sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int col0 = blockIdx.x * NT;
  const int row0 = blockIdx.y * kTailRows;
  const int nkc = h.dimp / kTailChunk;
  const int rowbytes = kQ4 ? h.dim / 2 : h.dim;
  const unsigned char* W = static_cast<const unsigned char*>(h.q);

  auto load = [&](int st, int kc) {
    unsigned char* A = sm + st * C::STAGE;
    unsigned char* B = A + C::A_BYTES;
    unsigned char* WS = B + C::B_BYTES;
    unsigned char* XS = WS + C::WS_BYTES;
    for (int id = tid; id < kTailRows * C::AU; id += kTailThreads) {
      const int r = id / C::AU, u = id % C::AU;
      const int off = kc * (C::AU * 16) + u * 16;
      const bool ok = row0 + r < h.vocab && off < rowbytes;
      const unsigned char* src = ok ? W + static_cast<size_t>(row0 + r) * rowbytes + off : W;
      const int su = kQ4 ? (u ^ ((r >> 1) & 3)) : (u ^ (r & 7));
      cp_async16_zfill(A + r * (C::AU * 16) + su * 16, src, ok);
    }
    for (int id = tid; id < NT * 8; id += kTailThreads) {
      const int c = id >> 3, u = id & 7;
      const bool ok = col0 + c < a.n;
      const int8_t* src = ok ? a.xq + static_cast<size_t>(col0 + c) * h.dimp + kc * kTailChunk + u * 16 : a.xq;
      cp_async16_zfill(B + c * kTailChunk + ((u ^ (c & 7)) << 4), src, ok);
    }
    if (tid < kTailRows) {
      const bool ok = row0 + tid < h.vocab;
      const uint16_t* src = ok ? h.s + static_cast<size_t>(row0 + tid) * h.nbp + kc * 4 : h.s;
      cp_async8_zfill(WS + tid * 8, src, ok);
    } else if (tid < kTailRows + NT) {
      const int c = tid - kTailRows;
      const bool ok = col0 + c < a.n;
      const float* src = ok ? a.xs + static_cast<size_t>(col0 + c) * h.nbp + kc * 4 : a.xs;
      cp_async16_zfill(XS + c * 16, src, ok);
    }
  };

  const int wm = warp % C::WARPS_M, wn = warp / C::WARPS_M;
  float2 acc[C::MI][C::NI][2];  // [..][..][0]: row g, tokens 2t, 2t+1; [1]: row g + 8
#pragma unroll
  for (int mi = 0; mi < C::MI; ++mi)
#pragma unroll
    for (int ni = 0; ni < C::NI; ++ni) acc[mi][ni][0] = acc[mi][ni][1] = make_float2(0.0f, 0.0f);

#pragma unroll
  for (int s = 0; s < kTailStages - 1; ++s) {
    if (s < nkc) load(s, s);
    cp_async_commit();
  }
  for (int kc = 0; kc < nkc; ++kc) {
    cp_async_wait<kTailStages - 2>();
    __syncthreads();  // chunk kc visible to all; the stage of chunk kc-1 is free
    {
      const int nk = kc + kTailStages - 1;
      if (nk < nkc) load(nk % kTailStages, nk);
      cp_async_commit();
    }
    const unsigned char* A = sm + (kc % kTailStages) * C::STAGE;
    const unsigned char* B = A + C::A_BYTES;
    const unsigned char* WS = B + C::B_BYTES;
    const unsigned char* XS = WS + C::WS_BYTES;

    float wsf[C::MI][2][4];  // h2f(scale_w) of my rows, 4 blocks
#pragma unroll
    for (int mi = 0; mi < C::MI; ++mi)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int r = wm * C::WM + mi * 16 + (lane >> 2) + hh * 8;
        const uint2 raw = *reinterpret_cast<const uint2*>(WS + r * 8);
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
        wsf[mi][hh][0] = lo.x;
        wsf[mi][hh][1] = lo.y;
        wsf[mi][hh][2] = hi.x;
        wsf[mi][hh][3] = hi.y;
      }
    float2 xsf[C::NI][4];  // scale_x of my two token columns, 4 blocks
#pragma unroll
    for (int ni = 0; ni < C::NI; ++ni) {
      const int c = wn * C::WN + ni * 8 + 2 * (lane & 3);
      const float4 x0 = *reinterpret_cast<const float4*>(XS + c * 16);
      const float4 x1 = *reinterpret_cast<const float4*>(XS + (c + 1) * 16);
      xsf[ni][0] = make_float2(x0.x, x1.x);
      xsf[ni][1] = make_float2(x0.y, x1.y);
      xsf[ni][2] = make_float2(x0.z, x1.z);
      xsf[ni][3] = make_float2(x0.w, x1.w);
    }

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
      for (int mi = 0; mi < C::MI; ++mi)
#pragma unroll
        for (int ni = 0; ni < C::NI; ++ni) {
          int d[4];
          mma_block(d, af[mi], bf[ni][0], bf[ni][1]);
          const float2 neg = make_float2(-kMagic, -kMagic);
          const float2 f01 = __fadd2_rn(make_float2(__int_as_float(d[0]), __int_as_float(d[1])), neg);
          const float2 f23 = __fadd2_rn(make_float2(__int_as_float(d[2]), __int_as_float(d[3])), neg);
          const float w0 = wsf[mi][0][bi], w1 = wsf[mi][1][bi];
          const float2 c01 = __fmul2_rn(make_float2(w0, w0), xsf[ni][bi]);
          const float2 c23 = __fmul2_rn(make_float2(w1, w1), xsf[ni][bi]);
          acc[mi][ni][0] = __ffma2_rn(c01, f01, acc[mi][ni][0]);
          acc[mi][ni][1] = __ffma2_rn(c23, f23, acc[mi][ni][1]);
        }
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // transpose through shared memory: each token's 128 logits leave as one run
  float* ot = reinterpret_cast<float*>(sm);
#pragma unroll
  for (int mi = 0; mi < C::MI; ++mi)
#pragma unroll
    for (int ni = 0; ni < C::NI; ++ni) {
      const int r = wm * C::WM + mi * 16 + (lane >> 2);
      const int c = wn * C::WN + ni * 8 + 2 * (lane & 3);
      ot[c * C::OUT_LD + r] = acc[mi][ni][0].x;
      ot[(c + 1) * C::OUT_LD + r] = acc[mi][ni][0].y;
      ot[c * C::OUT_LD + r + 8] = acc[mi][ni][1].x;
      ot[(c + 1) * C::OUT_LD + r + 8] = acc[mi][ni][1].y;
    }
  __syncthreads();
  for (int id = tid; id < NT * kTailRows; id += kTailThreads) {
    const int c = id / kTailRows, r = id % kTailRows;
    if (col0 + c < a.n && row0 + r < h.vocab)
      a.logits[static_cast<long long>(col0 + c) * a.ld + row0 + r] = ot[c * C::OUT_LD + r];
  }
}

// ------------------------------------------------------------ F32 head ----
// One vocab row per thread, NT tokens per CTA, the activations staged k-major
// so that a token pair is one float2; per (row, token) the products are added
// in index order, each rounded, as the reference's dot_f32.  Scalar
// __fmul_rn / __fadd_rn: the packed float2 forms are fused into one FFMA2 by
// the compiler, which the reference's separate roundings forbid.
template <int NT>
__global__ void __launch_bounds__(kTailThreads) tail_head_f32_kernel(TailHead h, TailArgs a) {
  __shared__ __align__(16) float xt[kF32Chunk][NT];
  const int row = blockIdx.y * kTailThreads + threadIdx.x;
  const int col0 = blockIdx.x * NT;
  const float* w = static_cast<const float*>(h.q) + static_cast<size_t>(min(row, h.vocab - 1)) * h.dim;
  float2 acc[NT / 2];
#pragma unroll
  for (int j = 0; j < NT / 2; ++j) acc[j] = make_float2(0.0f, 0.0f);
  for (int k0 = 0; k0 < h.dim; k0 += kF32Chunk) {
    const int len = min(kF32Chunk, h.dim - k0);  // a multiple of 32
    __syncthreads();
    for (int id = threadIdx.x; id < NT * len; id += kTailThreads) {
      const int c = id / len, k = id % len;
      xt[k][c] = col0 + c < a.n ? a.xb[static_cast<long long>(col0 + c) * h.dimp + k0 + k] : 0.0f;
    }
    __syncthreads();
    for (int k = 0; k < len; k += 4) {
      const float4 wv = *reinterpret_cast<const float4*>(w + k0 + k);
      const float we[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
#pragma unroll
        for (int j = 0; j < NT / 2; ++j) {
          const float2 xv = *reinterpret_cast<const float2*>(&xt[k + e][2 * j]);
          acc[j].x = __fadd_rn(acc[j].x, __fmul_rn(we[e], xv.x));
          acc[j].y = __fadd_rn(acc[j].y, __fmul_rn(we[e], xv.y));
        }
      }
    }
  }
  if (row >= h.vocab) return;
#pragma unroll
  for (int j = 0; j < NT / 2; ++j) {
    if (col0 + 2 * j < a.n) a.logits[static_cast<long long>(col0 + 2 * j) * a.ld + row] = acc[j].x;
    if (col0 + 2 * j + 1 < a.n) a.logits[static_cast<long long>(col0 + 2 * j + 1) * a.ld + row] = acc[j].y;
  }
}

template <int NT, bool kQ4>
cudaError_t launch_head_q(const TailHead& h, const TailArgs& a, cudaStream_t s) {
  using C = HeadCfg<NT, kQ4>;
  const cudaError_t e =
      cudaFuncSetAttribute(tail_head_q_kernel<NT, kQ4>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const dim3 grid((a.n + NT - 1) / NT, (h.vocab + kTailRows - 1) / kTailRows);
  tail_head_q_kernel<NT, kQ4><<<grid, kTailThreads, C::SMEM, s>>>(h, a);
  return cudaGetLastError();
}

template <bool kQ4>
cudaError_t launch_head_q_nt(const TailHead& h, const TailArgs& a, cudaStream_t s) {
  if (a.n <= 8) return launch_head_q<8, kQ4>(h, a, s);
  if (a.n <= 16) return launch_head_q<16, kQ4>(h, a, s);
  if (a.n <= 32) return launch_head_q<32, kQ4>(h, a, s);
  return launch_head_q<64, kQ4>(h, a, s);
}

template <int NT>
cudaError_t launch_head_f32(const TailHead& h, const TailArgs& a, cudaStream_t s) {
  const dim3 grid((a.n + NT - 1) / NT, (h.vocab + kTailThreads - 1) / kTailThreads);
  tail_head_f32_kernel<NT><<<grid, kTailThreads, 0, s>>>(h, a);
  return cudaGetLastError();
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

}  // namespace

size_t tail_scratch_bytes(const TailHead& h, int n) {
  const size_t rows = static_cast<size_t>(n);
  if (h.dtype == kTailF32) return align256(rows * h.dimp * 4);
  return align256(rows * h.dimp) + align256(rows * h.nbp * 4);
}

void tail_scratch_attach(const TailHead& h, int n, void* base, TailArgs& a) {
  unsigned char* p = static_cast<unsigned char*>(base);
  const size_t rows = static_cast<size_t>(n);
  a.xq = nullptr;
  a.xs = nullptr;
  a.xb = nullptr;
  if (h.dtype == kTailF32) {
    a.xb = reinterpret_cast<float*>(p);
    return;
  }
  a.xq = reinterpret_cast<int8_t*>(p);
  a.xs = reinterpret_cast<float*>(p + align256(rows * h.dimp));
}

int tail_kernels_per_call(const TailHead&) { return 2; }

cudaError_t launch_tail(const TailHead& h, const TailArgs& a, cudaStream_t s) {
  if (a.n <= 0) return cudaSuccess;
  tail_norm_kernel<<<(a.n + 7) / 8, kTailThreads, 0, s>>>(h, a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  switch (h.dtype) {
    case kTailQ8:
      return launch_head_q_nt<false>(h, a, s);
    case kTailQ4:
      return launch_head_q_nt<true>(h, a, s);
    default:
      return a.n <= 8 ? launch_head_f32<8>(h, a, s) : launch_head_f32<16>(h, a, s);
  }
}

}  // namespace vb
