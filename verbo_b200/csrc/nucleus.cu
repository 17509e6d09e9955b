// Streaming full-vocabulary path of Sampler::pick (src/sampler.cpp:71-108 with
// top_k == 0 or top_k >= vocab): the full sort, the softmax over every
// column, the top-p cutoff and the inverse-CDF draw, without sorting and with
// every logits row read from HBM once.
//
// Three streaming passes, each a kernel over every (row, slice of <=
// kSliceCols columns) with one CTA per slice and no CTA ever waiting for
// another, then one resolve CTA per row:
//
//   A  streams the slice from HBM and publishes its maximum and its
//                 smallest finite value (row atomics);
//   B  takes the row maximum M and builds an exact histogram of the
//                 slice's masses exp((v - M) / temp) over fine cells of
//                 x = (v - M) / temp.  The row's last slice to finish (a
//                 per-row counter) merges the slices' histograms and places the
//                 top-p cutoff (src/sampler.cpp:92-100) and the draw (:101-108)
//                 in one or two cells each, and the min-p boundary
//                 (:86-91) in the cells around x = ln(min_p);
//   C  gathers the slice's members of those cells;
//   R  resolves the pick among the row's members with the reference's fp64
//                 weights, in the reference's order.
//
// Rows go in chunks of kChunkRows (A, B, C, R kernels per chunk); each pass
// only reads what an earlier kernel wrote, so the kernels need no waits, and
// each has the resources its pass needs: the A pass, a plain stream, runs at
// full occupancy.  A single fused kernel running the passes of consecutive
// chunks side by side was slower: its CTAs all carried the largest pass's
// registers and shared memory.
//
// Exact masses without an exponential per column: cell j holds the columns
// whose x rounds to -j 2^-K; with r = x + j 2^-K (|r| <= 2^-(K+1)),
// exp(x) = exp(-j 2^-K) (1 + e(r)), e(r) = r + r^2/2 + r^3/6 evaluated in fp32
// and summed per cell in fixed point (2^-(K+22) units) with 32-bit shared
// atomics; the merge applies exp(-j 2^-K) once per cell in fp64.  Cumulative
// masses are within a few 1e-9 of the reference's sequential fp64 sums
// (kDelta bounds it), and the members of the cells where the decisions fall
// are resolved with exp((double)(v - M) / temp) as the reference computes it.
//
// Rows this path cannot settle exactly (a non-finite maximum, a cell holding
// more columns than its fixed-point sum allows, a decision outside the cells,
// too many members) are listed for the staged cluster kernel of kernels.cu,
// which launch_nucleus runs next on the same stream.
//
#include <algorithm>
#include <cstdint>

#include "device.cuh"
#include "kernels.cuh"
#include "rowdev.cuh"

namespace vb {
namespace nuc {

constexpr int NT = 256;
constexpr int kW = NT / 32;
constexpr int kSliceCols = 32768;    // columns of one slice (at most)
constexpr int kChunkRows = 2048;     // rows per B / C launch (their scratch)
constexpr int kCells = 2048;         // histogram capacity
constexpr int kCellTarget = 1024;    // the row's x-range is spread over about this many cells
constexpr int kKMin = 6;             // cells at most 2^-6 wide: |r| <= 2^-7
constexpr int kKMax = 20;
constexpr unsigned kCellCap = 1000;  // columns per cell and slice that keep the fixed-point sum exact
constexpr int kMemberCap = 2048;     // members gathered for the decisions
constexpr int kSubBins = NT;         // sub-bins of the resolve step
constexpr double kDelta = 4e-9;      // bound on the histogram's cumulative error, relative to the row's sum
constexpr unsigned kMagic23 = 0x4B400000u;  // bits of 1.5 * 2^23
constexpr int kQFix = 44;            // fixed-point fraction bits of the min-p boundary's mass (weights <= 1)
constexpr int kQCap = 1024;          // columns of the min-p boundary cells one C slice may hold

__device__ unsigned g_nuc_status;

// ------------------------------------------------------------ the grid ----
// Cells of x = (v - M) * (1 / temp) of width 2^-K: cell j (0 <= j <= ncr)
// holds the x that round to -j 2^-K.  A column whose x rounds below -ncr 2^-K
// (mass below e^-31 of the maximum's, or weight 0 for -inf / NaN) is
// "underflow": it only adds to the row's sum, and the B pass counts it in a
// trash cell ncr + 1 (x is clamped there before rounding).
struct Grid {
  float M, ih, il;   // 1 / temp = ih + il (fp32 pair)
  float magic;       // 1.5 * 2^(23 - K): adding it rounds to a multiple of 2^-K
  float xcut;        // -(ncr + 1) 2^-K: x is clamped to it before rounding (the trash cell)
  float two_s;       // 2^S, S = K + 22
  unsigned magic_bits;
  int K, S, ncr;
};

__device__ Grid make_grid(float M, float mlo, float temp) {
  Grid g;
  g.M = M;
  const double it = 1.0 / static_cast<double>(temp);
  g.ih = static_cast<float>(it);
  g.il = static_cast<float>(it - static_cast<double>(g.ih));
  const double xr = (static_cast<double>(M) - static_cast<double>(mlo)) * it;  // >= 0
  int K = kKMax;
  if (xr > 0.0) K = max(kKMin, min(kKMax, static_cast<int>(floor(log2((kCellTarget - 1) / xr)))));
  g.K = K;
  g.S = K + 22;
  g.ncr = static_cast<int>(fmin(floor(ldexp(xr, K)) + 2.0, static_cast<double>(kCells - 2)));
  g.xcut = static_cast<float>(-ldexp(static_cast<double>(g.ncr) + 1.0, -K));
  g.magic = ldexpf(1.5f, 23 - K);
  g.magic_bits = __float_as_uint(g.magic);
  g.two_s = ldexpf(1.0f, g.S);
  return g;
}

// d = v - M in fp32 as the reference rounds it (src/sampler.cpp:81) and
// x = d / temp in fp32, monotone in v; the same expressions everywhere.  A NaN
// v gives NaN (never in a cell), -0 the same as +0.
__device__ __forceinline__ float xof(float v, const Grid& g, float* d_out) {
  const float d = __fsub_rn(v, g.M);
  *d_out = d;
  return __fmul_rn(d, g.ih);
}
// Cell of x: x clamped to xcut (NaN too), then rounded to the grid; cells
// above ncr are underflow.  *t_out = the rounded x + magic.  The packed form in
// run_b computes the same bits as -(clamped x) rounded with -magic.
__device__ __forceinline__ int cell_of(float xh, const Grid& g, float* t_out) {
  const float t = __fadd_rn(fmaxf(xh, g.xcut), g.magic);
  *t_out = t;
  return static_cast<int>(g.magic_bits - __float_as_uint(t));
}
// Cell of a column value, or -1 for underflow.
__device__ __forceinline__ int cell_of_v(float v, const Grid& g) {
  float d, t;
  const int c = cell_of(xof(v, g, &d), g, &t);
  return c <= g.ncr ? c : -1;
}

// ---------------------------------------------- packed fp32x2 (sm_100) ----
// Two fp32 lanes in one 64-bit register; explicit .rn so that ptxas never
// contracts a multiply and an add into one rounding (the cell of a column
// must be the same in every pass).
typedef unsigned long long f2;
__device__ __forceinline__ f2 f2pk(float lo, float hi) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2up(f2 v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  f2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
  f2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  f2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// --------------------------------------------------------- the scratch ----
struct RowState {
  unsigned maxkey;      // ord32 of the row maximum (atomicMax)
  unsigned minkey_inv;  // ~ord32 of the smallest finite value (atomicMax); 0 = none
  unsigned cnt2;        // B slices done
  unsigned pad;
};
struct SliceSum {
  unsigned ucount;   // underflow columns
  unsigned crowded;  // a cell above kCellCap columns
  double umass;      // approximate mass of the underflow columns
};
// What the B merge leaves for the C kernel (per row of the chunk).
struct Targets {
  int fail;            // the row goes to the staged kernel
  int use_p;           // a top-p cutoff may decide the kept prefix
  int use_m;           // min-p: 0 none, 1 its boundary in cells [Q0, Q1], 2 it keeps every cell
  int A0, A1, B0, B1;  // cells of the cutoff and of the draw
  int Q0, Q1;          // cells of the min-p boundary (use_m == 1)
  float a_lo, a_hi, b_lo, b_hi;  // value intervals holding their members
  float q_lo, q_hi;
  unsigned cut_before;  // columns before A0
  unsigned q_before;    // columns before Q0 (use_m == 2: in every cell)
  double q_base;        // mass before Q0 (use_m == 2: of every cell)
  // columns of [Q0, Q1] with weight >= min_p, counted by the C slices
  // (atomics): their number, mass in 2^-kQFix units (exact, in any order),
  // largest key; and the smallest key of cell 0 (the first column)
  unsigned q_n, q_over;  // q_over: a slice had more than kQCap of them (the row goes to the staged kernel)
  unsigned long long q_mass, q_last, q_first;
  unsigned nmem;        // members gathered (C slices, atomic)
  double cut_base, draw_base;  // cumulative mass before A0 / B0
  double S, tp, u;
  unsigned long long s1, s0;   // the row's RNG state after this pick's draw
};

struct NucArgs {
  RowArgs a;
  int ns;            // slices per row
  int slice;         // columns per slice (multiple of 4)
  int rowa, rowb, rowc;  // first row of this launch's A, B, C chunk
  int na, nb, nc;        // rows of each (0: the phase has no chunk)
  unsigned* fb_count;   // rows listed for the staged kernel
  RowState* rs;         // [rows]
  int* fb_list;         // [rows]
  SliceSum* sums;       // [2 kChunkRows][ns]   (slot = row mod 2 kChunkRows)
  uint2* cells;         // [2 kChunkRows][ns][kCells]: (count, sum of the fixed-point words)
  Targets* tg;          // [2 kChunkRows]
  unsigned long long* members;  // [2 kChunkRows][kMemberCap] keys
};

// Scratch layout; the first `zero_bytes` are cleared before every call.
struct Layout {
  size_t off_rs, zero_bytes, off_fb, off_sum, off_cells, off_tg, off_mem, bytes;
};
static size_t up256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }
static Layout layout(int rows, int ns) {
  const size_t cr = static_cast<size_t>(std::min(rows, kChunkRows));
  Layout l;
  l.off_rs = 256;
  l.zero_bytes = l.off_rs + sizeof(RowState) * static_cast<size_t>(rows);
  l.off_fb = up256(l.zero_bytes);
  l.off_sum = up256(l.off_fb + sizeof(int) * static_cast<size_t>(rows));
  l.off_cells = up256(l.off_sum + sizeof(SliceSum) * cr * static_cast<size_t>(ns));
  l.off_tg = up256(l.off_cells + sizeof(uint2) * kCells * cr * static_cast<size_t>(ns));
  l.off_mem = up256(l.off_tg + sizeof(Targets) * cr);
  l.bytes = up256(l.off_mem + sizeof(unsigned long long) * kMemberCap * cr);
  return l;
}

// --------------------------------------------------------- streaming ------
// f(value, column) for every column of [0, n) of src, each once: a scalar head
// up to the first 16-byte boundary, the body in 16-byte loads (kU in flight
// per thread), a scalar tail.  kHbm: streaming loads that keep the lines in
// L2 for the later passes; otherwise L2-only loads.
template <int kU, bool kHbm, class F>
__device__ __forceinline__ void each_col(const float* src, int n, F&& f) {
  const uintptr_t addr = reinterpret_cast<uintptr_t>(src);
  int h = static_cast<int>(((16 - (addr & 15)) & 15) >> 2);
  if (h > n) h = n;
  if (static_cast<int>(threadIdx.x) < h) f(src[threadIdx.x], static_cast<int>(threadIdx.x));
  const float4* b4 = reinterpret_cast<const float4*>(src + h);
  const int n4 = (n - h) >> 2;
  int q = threadIdx.x;
  for (; q + (kU - 1) * NT < n4; q += kU * NT) {
    float4 t[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) t[u] = kHbm ? ld_stream(b4 + q + u * NT) : __ldcg(b4 + q + u * NT);
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int j = h + 4 * (q + u * NT);
      f(t[u].x, j);
      f(t[u].y, j + 1);
      f(t[u].z, j + 2);
      f(t[u].w, j + 3);
    }
  }
  for (; q < n4; q += NT) {
    const float4 t = kHbm ? ld_stream(b4 + q) : __ldcg(b4 + q);
    const int j = h + 4 * q;
    f(t.x, j);
    f(t.y, j + 1);
    f(t.z, j + 2);
    f(t.w, j + 3);
  }
  for (int j = h + 4 * n4 + threadIdx.x; j < n; j += NT) f(src[j], j);
}

// Software-pipelined traversal for the compute-carrying passes: rounds of kU
// 16-byte streaming loads per thread, the next round issued before the
// current one is processed, so a round's latency overlaps the previous
// round's work.  f4(float4, column of .x) for the aligned body, f1(value,
// column) for the scalar head and tail.
template <int kU, class F4, class F1>
__device__ __forceinline__ void each_col_pipe(const float* src, int n, F4&& f4, F1&& f1) {
  const uintptr_t addr = reinterpret_cast<uintptr_t>(src);
  int h = static_cast<int>(((16 - (addr & 15)) & 15) >> 2);
  if (h > n) h = n;
  if (static_cast<int>(threadIdx.x) < h) f1(src[threadIdx.x], static_cast<int>(threadIdx.x));
  const float4* b4 = reinterpret_cast<const float4*>(src + h);
  const int n4 = (n - h) >> 2;
  constexpr int R = kU * NT;  // vectors per round
  const int rounds = n4 / R;  // full rounds
  float4 cur[kU], nxt[kU];
  if (rounds > 0) {
#pragma unroll
    for (int u = 0; u < kU; ++u) cur[u] = ld_stream(b4 + threadIdx.x + u * NT);
  }
  for (int r = 0; r < rounds; ++r) {
    const int q = r * R + threadIdx.x;
    if (r + 1 < rounds) {
#pragma unroll
      for (int u = 0; u < kU; ++u) nxt[u] = ld_stream(b4 + q + R + u * NT);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) f4(cur[u], h + 4 * (q + u * NT));
#pragma unroll
    for (int u = 0; u < kU; ++u) cur[u] = nxt[u];
  }
  for (int q = rounds * R + threadIdx.x; q < n4; q += NT) f4(ld_stream(b4 + q), h + 4 * q);
  for (int j = h + 4 * n4 + threadIdx.x; j < n; j += NT) f1(src[j], j);
}

// -------------------------------------------------------------- shared ----
struct Shared {
  NucArgs p;  // the kernel parameters, copied here so that every function reads them from shared memory
  DevOpts o;
  Grid g;     // the grid of the row at hand
  unsigned mbase;  // C items: first member slot reserved by this CTA
  int kind, row, slice;
  int last;
  int flag;
  float wsf[kW];
  unsigned wsu[kW];
  unsigned wsc[kW];
  double wsd[kW];
  int c_lo, c_hi, d_lo, d_hi;
  unsigned nmem;
  int sb;  // resolve: target sub-bin
  double sb_base;
  unsigned sb_n, sb_cnt_before;
  int r_found;
  unsigned long long r_key;
  double r_cum;
  unsigned r_rank;
  // C items: the CTA's count of the min-p boundary (see Targets)
  unsigned q_n, q_cnt;
  unsigned long long q_mass, q_last, q_first;
};

// Dynamic shared memory: B items [kCells] counts + [kCells] fixed-point sums;
// the B merge [kCells] doubles + [kCells] counts; the C merge the member keys,
// their weights, a sort buffer and the sub-bins.
constexpr size_t kHistBytes = static_cast<size_t>(kCells) * 8;
constexpr size_t kCumBytes = static_cast<size_t>(kCells) * 12;
constexpr size_t kMemberBytes = static_cast<size_t>(kMemberCap) * 24 + static_cast<size_t>(kSubBins) * 12;
constexpr size_t kBSmem = std::max(kHistBytes, kCumBytes);         // B pass + its row merge
constexpr size_t kCSmem = static_cast<size_t>(kMemberCap + kQCap) * 8;  // C pass: members, min-p boundary keys
constexpr size_t kRSmem = kMemberBytes;                             // resolve
constexpr int kBBlocks = 4, kCBlocks = 6;                           // resident CTAs per SM aimed at

template <class T>
__device__ __forceinline__ T bsum(T x, T* ws) {
  x = warp_sum(x);
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = x;
  __syncthreads();
  T r = ws[0];
#pragma unroll
  for (int i = 1; i < kW; ++i) r += ws[i];
  __syncthreads();
  return r;
}

// Block scan of (w, c) pairs in thread order: exclusive prefixes and totals.
__device__ __noinline__ void bscan(double w, unsigned c, Shared& sh, double* wpre, unsigned* cpre, double* wtot,
                                   unsigned* ctot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double wi = w;
  unsigned ci = c;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, wi, off);
    const unsigned cy = __shfl_up_sync(0xffffffffu, ci, off);
    if (lane >= off) {
      wi += y;
      ci += cy;
    }
  }
  if (lane == 31) {
    sh.wsd[warp] = wi;
    sh.wsu[warp] = ci;
  }
  __syncthreads();
  double wp = 0.0, wt = 0.0;
  unsigned cp = 0, ct = 0;
  for (int i = 0; i < kW; ++i) {
    if (i < warp) {
      wp += sh.wsd[i];
      cp += sh.wsu[i];
    }
    wt += sh.wsd[i];
    ct += sh.wsu[i];
  }
  __syncthreads();
  *wpre = wp + wi - w;
  *cpre = cp + ci - c;
  *wtot = wt;
  *ctot = ct;
}

// The row's grid from its published maximum and smallest finite value.
__device__ __forceinline__ Grid row_grid(const RowState* st, float temp) {
  const unsigned mk = __ldcg(&st->maxkey);
  const unsigned nk = __ldcg(&st->minkey_inv);
  const float M = unord32(mk);
  const float mlo = nk != 0u ? unord32(~nk) : M;
  return make_grid(M, isfinite(M) && isfinite(mlo) ? mlo : M, temp);
}

// The reference's weight of a column (src/sampler.cpp:81), fp64.
__device__ __noinline__ double ref_weight(float v, float M, double temp_d) {
  return exp(__ddiv_rn(static_cast<double>(__fsub_rn(canon(v), M)), temp_d));
}

__device__ __forceinline__ void to_fallback(const NucArgs& p, int row) {
  const unsigned i = atomicAdd(p.fb_count, 1u);
  p.fb_list[i] = row;
}

// ------------------------------------------------------------- A items ----
__device__ __noinline__ void run_a(int row, int s, Shared& sh) {
  const NucArgs& p = sh.p;
  const RowArgs& a = p.a;
  const int lo = s * p.slice;
  const int n = min(p.slice, a.ncols - lo);
  const float* src = a.logits + static_cast<long long>(row) * a.ld + lo;
  const float ninf = -__int_as_float(0x7f800000), pinf = __int_as_float(0x7f800000);
  float mx = ninf, mn = pinf;
  each_col<8, true>(src, n, [&](float v, int) {
    mx = fmaxf(mx, v);                    // a NaN never wins
    mn = fminf(mn, v > ninf ? v : pinf);  // finite (and +inf) values only
  });
  mx = warp_max(mx);
  mn = warp_min(mn);
  if ((threadIdx.x & 31) == 0) {
    sh.wsf[threadIdx.x >> 5] = mx;
    sh.wsu[threadIdx.x >> 5] = __float_as_uint(mn);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < kW; ++i) {
      mx = fmaxf(mx, sh.wsf[i]);
      mn = fminf(mn, __uint_as_float(sh.wsu[i]));
    }
    RowState* st = p.rs + row;
    atomicMax(&st->maxkey, ord32(canon(mx)));
    if (mn < pinf) atomicMax(&st->minkey_inv, ~ord32(canon(mn)));
  }
  __syncthreads();
}

// ------------------------------------------------------------- B items ----
__device__ __noinline__ void merge_b(int row, unsigned char* smem, Shared& sh);

__device__ __noinline__ void run_b(int row, int s, unsigned char* smem, Shared& sh) {
  const NucArgs& p = sh.p;
  const DevOpts& o = sh.o;
  const RowArgs& a = p.a;
  RowState* st = p.rs + row;
  const int slot = row % kChunkRows;
  unsigned* cnt = reinterpret_cast<unsigned*>(smem);
  unsigned* esm = cnt + kCells;
  // the grid (thread 0, an L2 round trip) while every cell is cleared
  if (threadIdx.x == 0) sh.g = row_grid(st, o.temp);
  for (int c = threadIdx.x; c < kCells; c += NT) {
    cnt[c] = 0u;
    esm[c] = 0u;
  }
  __syncthreads();
  const Grid g = sh.g;
  const int nc = g.ncr + 1;  // cells 0..ncr, and nc: the trash cell (ncr <= kCells - 2)
  const int lo = s * p.slice;
  const int n = min(p.slice, a.ncols - lo);
  const float* src = a.logits + static_cast<long long>(row) * a.ld + lo;
  unsigned uc = 0;
  float um = 0.0f;
  const float ninf = -__int_as_float(0x7f800000);
  if (isfinite(g.M)) {
    // Two columns at a time in packed fp32x2, without a branch: nx = -x (the
    // negated product rounds like the product), clamped to -xcut (underflow,
    // -inf and NaN land in the trash cell ncr + 1), nt = -(nx + magic ...) =
    // -t, so the cell is the scalar cell_of's; ngg = -(grid point), r = x -
    // grid point in one rounding, e(r), y = magic23 + round(e 2^S).
    const f2 nM = f2pk(-g.M, -g.M), nih = f2pk(-g.ih, -g.ih), ih = f2pk(g.ih, g.ih), il = f2pk(g.il, g.il);
    const f2 nmag = f2pk(-g.magic, -g.magic), mag = f2pk(g.magic, g.magic), tws = f2pk(g.two_s, g.two_s);
    const f2 c6 = f2pk(0.16666667f, 0.16666667f), c2 = f2pk(0.5f, 0.5f), c1 = f2pk(1.0f, 1.0f);
    const f2 m23 = f2pk(12582912.0f, 12582912.0f);
    const float hi = -g.xcut;
    const unsigned kidx = g.magic_bits + 0x80000000u;  // cell = kidx - bits(-t)
    auto two = [&](float va, float vb) {
      const f2 d = add2(f2pk(va, vb), nM);
      float na, nb;
      f2up(mul2(d, nih), na, nb);
      const f2 nt = add2(f2pk(fminf(na, hi), fminf(nb, hi)), nmag);
      const f2 ngg = add2(nt, mag);
      f2 r = fma2(d, ih, ngg);
      r = fma2(d, il, r);
      const f2 y = fma2(mul2(r, fma2(r, fma2(r, c6, c2), c1)), tws, m23);
      float ta, tb, ya, yb;
      f2up(nt, ta, tb);
      f2up(y, ya, yb);
      const unsigned ia = kidx - __float_as_uint(ta), ib = kidx - __float_as_uint(tb);
      atomicAdd(cnt + ia, 1u);
      atomicAdd(esm + ia, __float_as_uint(ya));
      atomicAdd(cnt + ib, 1u);
      atomicAdd(esm + ib, __float_as_uint(yb));
    };
    each_col_pipe<4>(src, n, [&](const float4& v, int) {
      two(v.x, v.y);
      two(v.z, v.w);
    }, [&](float v, int) { two(v, ninf); });  // head and tail: the -inf partner lands in the trash cell
  }
  __syncthreads();
  // underflow columns (rare): their count and approximate mass, in a second
  // pass over the slice (the trash cell also holds the weight-0 columns and
  // the head / tail partners, which are told apart here)
  if (isfinite(g.M) && cnt[nc] != 0u) {
    each_col<4, true>(src, n, [&](float v, int) {
      float d, t;
      const float xh = xof(v, g, &d);
      if (d > ninf && cell_of(xh, g, &t) > g.ncr) {
        ++uc;
        um += __expf(xh);
      }
    });
  }
  __syncthreads();
  // flush cells [0, nc) of this slice and its summary into the row's slot
  uint2* out = p.cells + (static_cast<long long>(slot) * p.ns + s) * kCells;
  unsigned crowded = 0;
  for (int c = threadIdx.x; c < nc; c += NT) {
    const uint2 v = make_uint2(cnt[c], esm[c]);
    crowded |= v.x > kCellCap ? 1u : 0u;
    __stcg(out + c, v);
  }
  // the slice's summary in one reduction round (warp sums, then thread 0)
  {
    const unsigned wu = warp_sum(uc), wc = warp_sum(crowded);
    const double wm = warp_sum(static_cast<double>(um));
    if ((threadIdx.x & 31) == 0) {
      sh.wsu[threadIdx.x >> 5] = wu;
      sh.wsc[threadIdx.x >> 5] = wc;
      sh.wsd[threadIdx.x >> 5] = wm;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    SliceSum v;
    v.ucount = 0;
    v.crowded = 0;
    v.umass = 0.0;
    for (int i = 0; i < kW; ++i) {
      v.ucount += sh.wsu[i];
      v.crowded += sh.wsc[i];
      v.umass += sh.wsd[i];
    }
    p.sums[static_cast<long long>(slot) * p.ns + s] = v;
    __threadfence();
    const unsigned old = atomicAdd(&st->cnt2, 1u);
    sh.last = old == static_cast<unsigned>(p.ns - 1);
    __threadfence();
  }
  __syncthreads();
  if (sh.last) merge_b(row, smem, sh);
}

// The row's merged histogram: per-cell cumulative masses, the cells of the
// top-p cutoff (src/sampler.cpp:92-100) and of the draw (:101-108), and the
// value intervals holding their members, published for the C items.
__device__ __noinline__ void merge_b(int row, unsigned char* smem, Shared& sh) {
  const NucArgs& p = sh.p;
  const DevOpts& o = sh.o;
  const Grid& g = sh.g;
  const RowArgs& a = p.a;
  const int slot = row % kChunkRows;
  const int nc = g.ncr + 1;
  double* cum = reinterpret_cast<double*>(smem);             // [kCells] inclusive cumulative mass
  unsigned* cnt = reinterpret_cast<unsigned*>(cum + kCells);  // [kCells] columns before each cell
  const uint2* cells = p.cells + static_cast<long long>(slot) * p.ns * kCells;
  const SliceSum* sums = p.sums + static_cast<long long>(slot) * p.ns;
  if (threadIdx.x == 0) {
    int f = !isfinite(g.M);
    for (int s = 0; s < p.ns; ++s) f |= __ldcg(&sums[s].crowded) != 0u;
    sh.flag = f;
    sh.c_lo = sh.c_hi = sh.d_lo = sh.d_hi = nc;
  }
  __syncthreads();
  // per-cell sums over the slices: thread t takes the cell pairs 2t, 2t + 1
  // (+ 2 NT, ...) and issues the 16-byte loads of two slices before adding
  // any of them
  const double unit = ldexp(1.0, -g.S);
  {
    constexpr int KP = kCells / (2 * NT);  // cell pairs per thread
    constexpr int SB = 2;                  // slices per batch of loads
    unsigned n[2 * KP];
    long long e[2 * KP];
#pragma unroll
    for (int k = 0; k < 2 * KP; ++k) {
      n[k] = 0;
      e[k] = 0;
    }
    const uint4* cells4 = reinterpret_cast<const uint4*>(cells);
    for (int s0 = 0; s0 < p.ns; s0 += SB) {
      uint4 v[SB][KP];
#pragma unroll
      for (int b = 0; b < SB; ++b)
#pragma unroll
        for (int k = 0; k < KP; ++k) {
          const int c = 2 * (threadIdx.x + k * NT);
          v[b][k] = s0 + b < p.ns && c < nc ? __ldcg(cells4 + (static_cast<long long>(s0 + b) * kCells + c) / 2)
                                            : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
      for (int b = 0; b < SB; ++b)
#pragma unroll
        for (int k = 0; k < KP; ++k) {
          n[2 * k] += v[b][k].x;
          e[2 * k] += static_cast<int>(v[b][k].y - v[b][k].x * kMagic23);
          n[2 * k + 1] += v[b][k].z;
          e[2 * k + 1] += static_cast<int>(v[b][k].w - v[b][k].z * kMagic23);
        }
    }
#pragma unroll
    for (int k = 0; k < 2 * KP; ++k) {
      const int c = 2 * (threadIdx.x + (k >> 1) * NT) + (k & 1);
      if (c < nc) {
        cum[c] = n[k] ? exp(-ldexp(static_cast<double>(c), -g.K)) *
                            (static_cast<double>(n[k]) + static_cast<double>(e[k]) * unit)
                      : 0.0;
        cnt[c] = n[k];
      }
    }
  }
  __syncthreads();
  // thread t owns cells [c0, c1) for the scans
  const int cpt = (nc + NT - 1) / NT;
  const int c0 = threadIdx.x * cpt, c1 = min(nc, c0 + cpt);
  double local = 0.0;
  unsigned lcnt = 0;
  for (int c = c0; c < c1; ++c) {
    local += cum[c];
    lcnt += cnt[c];
  }
  double U = 0.0;
  unsigned Uc = 0;
  for (int s = 0; s < p.ns; ++s) {
    U += __ldcg(&sums[s].umass);
    Uc += __ldcg(&sums[s].ucount);
  }
  double wpre, wtot;
  unsigned cpre, ctot;
  bscan(local, lcnt, sh, &wpre, &cpre, &wtot, &ctot);
  {
    double run = wpre;
    unsigned crun = cpre;
    for (int c = c0; c < c1; ++c) {
      run += cum[c];
      cum[c] = run;
      const unsigned n = cnt[c];
      cnt[c] = crun;
      crun += n;
    }
  }
  __syncthreads();
  const double S = wtot + U;  // the softmax normaliser (src/sampler.cpp:80-85)
  const double dl = kDelta * S;
  auto first_reach = [&](double x, int* outc) {  // first cell whose cumulative mass reaches x
    for (int c = c0; c < c1; ++c)
      if (cum[c] >= x) {
        atomicMin(outc, c);
        break;
      }
  };
  const bool use_p = o.top_p > 0.0f && o.top_p < 1.0f;
  const double tp = use_p ? static_cast<double>(o.top_p) * S : 0.0;
  if (use_p) {
    first_reach(tp - dl, &sh.c_lo);
    first_reach(tp + dl, &sh.c_hi);
  }
  // this pick's uniform (src/sampler.cpp:103)
  unsigned long long s1 = 0, s0 = 0;
  double u = 0.0;
  if (a.rng) {
    s1 = a.rng[2ll * row];
    s0 = a.rng[2ll * row + 1];
    u = rng_unit(s1, s0);
  }
  __syncthreads();
  int A0 = use_p ? sh.c_lo : nc, A1 = use_p ? sh.c_hi : -1;
  bool fail = sh.flag != 0;
  // min-p (src/sampler.cpp:86-91): the max's weight is exp(0) = 1, so the
  // kept prefix is every column with weight >= min_p, at least one; its
  // boundary lies in the cells around x* = ln(min_p), widened for the fp32
  // roundings of x.  use_m 2: x* lies below every cell and no column
  // underflows, so min-p keeps every cell.
  int use_m = 0, Q0 = nc, Q1 = -1;
  bool m_unsure = false;  // the boundary may reach the underflow columns
  if (o.min_p > 0.0f) {
    // the cells of x* -+ (a hundredth of a cell + a relative 1e-5), the
    // slack of the fp32 x against the exact d / temp (as in vbound below)
    const double xs = log(static_cast<double>(o.min_p));
    const double eps = ldexp(0.01, -g.K) + 1e-5 * fabs(xs);
    const double lo = rint(-ldexp(xs + eps, g.K)), hi = rint(-ldexp(xs - eps, g.K));
    if (lo > static_cast<double>(g.ncr)) {
      use_m = 2;
      m_unsure = Uc != 0;
    } else {
      use_m = 1;
      Q0 = static_cast<int>(fmax(lo, 0.0));
      Q1 = static_cast<int>(fmin(hi, static_cast<double>(g.ncr)));
      m_unsure = hi > static_cast<double>(g.ncr) && Uc != 0;
    }
  }
  const bool p_beyond = use_p && (A0 >= nc || A1 >= nc);  // the cutoff lies among the underflow columns
  // the ranges of each cut's running mass; the kept prefix is the shorter
  double lo_p = S, hi_p = S, lo_m = S, hi_m = S;
  if (use_p && !p_beyond) {
    lo_p = A0 > 0 ? cum[A0 - 1] : 0.0;
    hi_p = cum[A1];
  }
  if (use_m == 1) {
    lo_m = Q0 > 0 ? cum[Q0 - 1] : 0.0;
    hi_m = cum[Q1];
  } else if (use_m == 2) {
    lo_m = hi_m = wtot;
  }
  bool need_p = use_p && !p_beyond, need_m = use_m == 1;
  if (need_p && use_m == 1 && A0 > Q1) need_p = false;  // min-p keeps fewer columns for certain
  if (need_m && need_p && A1 < Q0) need_m = false;      // top-p does
  if (!need_p) lo_p = hi_p = S;
  if (!need_m && use_m == 1) lo_m = hi_m = S;
  if (p_beyond && !(use_m == 1 && !m_unsure)) fail = true;  // top-p may cut among the underflow columns
  if (m_unsure && !(need_p && A1 < Q0)) fail = true;     // so may min-p
  if (use_m == 2 && need_p) use_m = 0;                 // top-p cuts within the cells, before min-p
  if (use_m == 1 && !need_m) use_m = 0;
  if (!need_p) {
    A0 = nc;
    A1 = -1;
  }
  const double tot_lo = fmin(lo_p, lo_m), tot_hi = fmin(hi_p, hi_m);
  if (!fail && u * tot_hi + dl > wtot) fail = true;  // the draw may fall among the underflow columns
  if (!fail) {
    first_reach(u * tot_lo - dl, &sh.d_lo);
    first_reach(u * tot_hi + dl, &sh.d_hi);
  }
  __syncthreads();
  const int B0 = sh.d_lo, B1 = sh.d_hi;
  if (threadIdx.x == 0) {
    Targets* t = p.tg + slot;
    auto before = [&](int c) -> unsigned { return c < nc ? cnt[c] : ctot; };
    if (!fail && (B0 >= nc || B1 >= nc)) fail = true;
    if (!fail) {
      unsigned need = before(B1 + 1) - before(B0);
      if (A1 >= A0) need += before(A1 + 1) - before(A0);
      if (need > static_cast<unsigned>(kMemberCap)) fail = true;
    }
    t->fail = fail;
    if (!fail) {
      // value intervals holding every member of [A0, A1] and [B0, B1]: x of
      // the cells' outer edges, widened by a hundredth of a cell and a
      // relative 1e-5 for the fp32 roundings of x
      const double temp_d = static_cast<double>(o.temp);
      auto vbound = [&](int c, double side) -> float {
        const double xb = -ldexp(static_cast<double>(c) - 0.5 * side, -g.K);
        const double w = ldexp(0.01, -g.K) + 1e-5 * fabs(xb);
        return static_cast<float>(static_cast<double>(g.M) + (xb + side * w) * temp_d);
      };
      const bool pa = A1 >= A0;
      t->use_p = pa;
      t->use_m = use_m;
      t->A0 = A0;
      t->A1 = A1;
      t->B0 = B0;
      t->B1 = B1;
      t->Q0 = use_m == 1 ? Q0 : nc;
      t->Q1 = use_m == 1 ? Q1 : -1;
      t->a_lo = pa ? vbound(A1, -1.0) : __int_as_float(0x7f800000);
      t->a_hi = pa ? vbound(A0, 1.0) : -__int_as_float(0x7f800000);
      t->b_lo = vbound(B1, -1.0);
      t->b_hi = vbound(B0, 1.0);
      t->q_lo = use_m == 1 ? vbound(Q1, -1.0) : __int_as_float(0x7f800000);
      t->q_hi = use_m == 1 ? vbound(Q0, 1.0) : -__int_as_float(0x7f800000);
      t->cut_before = pa ? before(A0) : 0u;
      t->cut_base = pa && A0 > 0 ? cum[A0 - 1] : 0.0;
      t->q_before = use_m == 1 ? before(Q0) : ctot;
      t->q_base = use_m == 1 ? (Q0 > 0 ? cum[Q0 - 1] : 0.0) : wtot;
      t->q_n = 0;
      t->q_over = 0;
      t->q_mass = 0;
      t->q_last = 0;
      t->q_first = kNoKey;
      t->draw_base = B0 > 0 ? cum[B0 - 1] : 0.0;
      t->S = S;
      t->tp = tp;
      t->u = u;
      t->s1 = s1;
      t->s0 = s0;
    }
    t->nmem = 0;
  }
  __syncthreads();
}

// ------------------------------------------------------------- C items ----
// A column of the min-p boundary cells (src/sampler.cpp:86-91), after the
// scan: counted into the CTA's totals when its weight, as the reference
// computes it, reaches min_p (the max's weight is exp(0) = 1).
__device__ __forceinline__ void q_note(unsigned long long k, int c, float M, Shared& sh) {
  const double w = ref_weight(dval(k), M, static_cast<double>(sh.o.temp));
  if (w >= static_cast<double>(sh.o.min_p)) {
    atomicAdd(&sh.q_n, 1u);
    atomicAdd(&sh.q_mass, __double2ull_rn(ldexp(w, kQFix)));
    atomicMax(&sh.q_last, k);
  }
  if (c == 0) atomicMin(&sh.q_first, k);
}

// kMinP: the call has min-p, so rows may carry a min-p boundary to count; the
// form without it keeps the scan loop free of that bookkeeping.
template <bool kMinP>
__device__ __noinline__ void run_c(int row, int s, unsigned char* smem, Shared& sh) {
  const NucArgs& p = sh.p;
  const DevOpts& o = sh.o;
  const RowArgs& a = p.a;
  RowState* st = p.rs + row;
  const int ms = row % kChunkRows;
  const Targets* tg = p.tg + ms;
  const int fail = __ldcg(&tg->fail);
  if (!fail) {
    // the slice's members go to shared memory first, then to the row's list
    // with one reservation per CTA
    if (threadIdx.x == 0) sh.nmem = 0;
    __syncthreads();
    const Grid g = row_grid(st, o.temp);
    const int A0 = __ldcg(&tg->A0), A1 = __ldcg(&tg->A1), B0 = __ldcg(&tg->B0), B1 = __ldcg(&tg->B1);
    const int Q0 = kMinP ? __ldcg(&tg->Q0) : 0, Q1 = kMinP ? __ldcg(&tg->Q1) : -1;
    const float a_lo = __ldcg(&tg->a_lo), a_hi = __ldcg(&tg->a_hi);
    const float b_lo = __ldcg(&tg->b_lo), b_hi = __ldcg(&tg->b_hi);
    const float q_lo = kMinP ? __ldcg(&tg->q_lo) : 0.0f, q_hi = kMinP ? __ldcg(&tg->q_hi) : -1.0f;
    const bool use_a = A1 >= A0, use_q = kMinP && Q1 >= Q0;
    unsigned long long* loc = reinterpret_cast<unsigned long long*>(smem);  // [kMemberCap]
    const int lo = s * p.slice;
    const int n = min(p.slice, a.ncols - lo);
    const float* src = a.logits + static_cast<long long>(row) * a.ld + lo;
    const unsigned gid0 = static_cast<unsigned>(a.col_off + lo);
    unsigned long long* qloc = loc + kMemberCap;  // [kQCap] keys of the min-p boundary cells
    if (kMinP) {
      if (threadIdx.x == 0) {
        sh.q_n = 0;
        sh.q_cnt = 0;
        sh.q_mass = 0;
        sh.q_last = 0;
        sh.q_first = kNoKey;
      }
      __syncthreads();
    }
    auto test = [&](float v, int j) {
      if ((v >= a_lo && v <= a_hi) || (v >= b_lo && v <= b_hi) || (kMinP && v >= q_lo && v <= q_hi)) {
        const int c = cell_of_v(v, g);
        if (kMinP && c >= Q0 && c <= Q1) {
          const unsigned q = atomicAdd(&sh.q_cnt, 1u);
          if (q < static_cast<unsigned>(kQCap)) qloc[q] = dkey(v, gid0 + static_cast<unsigned>(j));
        }
        if ((c >= A0 && c <= A1) || (c >= B0 && c <= B1)) {
          const unsigned q = atomicAdd(&sh.nmem, 1u);
          if (q < static_cast<unsigned>(kMemberCap)) loc[q] = dkey(v, gid0 + static_cast<unsigned>(j));
        }
      }
    };
    // prefilter per 16-byte vector: the smallest distance of its columns to
    // each interval's midpoint (packed fp32x2), against the half-width widened
    // by a relative 1e-6 for the rounding of the distance
    const float ma = use_a ? 0.5f * (a_lo + a_hi) : __int_as_float(0x7f800000);
    const float ha = use_a ? 0.5f * (a_hi - a_lo) * (1.0f + 1e-6f) + 1e-30f : -1.0f;
    const float mb = 0.5f * (b_lo + b_hi), hb = 0.5f * (b_hi - b_lo) * (1.0f + 1e-6f) + 1e-30f;
    const float mq = use_q ? 0.5f * (q_lo + q_hi) : 0.0f;
    const float hq = use_q ? 0.5f * (q_hi - q_lo) * (1.0f + 1e-6f) + 1e-30f : -1.0f;
    const f2 nma = f2pk(-ma, -ma), nmb = f2pk(-mb, -mb), nmq = f2pk(-mq, -mq);
    each_col_pipe<4>(src, n, [&](const float4& v, int j) {
      const f2 v01 = f2pk(v.x, v.y), v23 = f2pk(v.z, v.w);
      float a0, a1, a2, a3, b0, b1, b2, b3;
      f2up(add2(v01, nma), a0, a1);
      f2up(add2(v23, nma), a2, a3);
      f2up(add2(v01, nmb), b0, b1);
      f2up(add2(v23, nmb), b2, b3);
      const float da = fminf(fminf(fabsf(a0), fabsf(a1)), fminf(fabsf(a2), fabsf(a3)));
      const float db = fminf(fminf(fabsf(b0), fabsf(b1)), fminf(fabsf(b2), fabsf(b3)));
      bool hit = da <= ha || db <= hb;
      if (kMinP && use_q) {  // min-p boundary cells (a uniform branch: one row per CTA)
        float q0, q1, q2, q3;
        f2up(add2(v01, nmq), q0, q1);
        f2up(add2(v23, nmq), q2, q3);
        hit |= fminf(fminf(fabsf(q0), fabsf(q1)), fminf(fabsf(q2), fabsf(q3))) <= hq;
      }
      if (hit) {
        test(v.x, j);
        test(v.y, j + 1);
        test(v.z, j + 2);
        test(v.w, j + 3);
      }
    }, test);
    __syncthreads();
    if (use_q) {  // the boundary's columns: weights and counts, out of the scan loop
      const unsigned qc = min(sh.q_cnt, static_cast<unsigned>(kQCap));
      for (unsigned i = threadIdx.x; i < qc; i += NT) {
        const unsigned long long k = qloc[i];
        float d, t;
        q_note(k, cell_of(xof(dval(k), g, &d), g, &t), g.M, sh);
      }
      __syncthreads();
    }
    const unsigned cnt = min(sh.nmem, static_cast<unsigned>(kMemberCap));
    if (threadIdx.x == 0) {
      sh.mbase = cnt ? atomicAdd(&p.tg[ms].nmem, sh.nmem) : 0u;
      if (use_q && sh.q_cnt > static_cast<unsigned>(kQCap)) atomicOr(&p.tg[ms].q_over, 1u);
      if (use_q) {  // the slice's count of the min-p boundary, one atomic per field
        Targets* tw = p.tg + ms;
        if (sh.q_n) {
          atomicAdd(&tw->q_n, sh.q_n);
          atomicAdd(&tw->q_mass, sh.q_mass);
          atomicMax(&tw->q_last, sh.q_last);
        }
        if (sh.q_first != kNoKey) atomicMin(&tw->q_first, sh.q_first);
      }
    }
    __syncthreads();
    unsigned long long* mem = p.members + static_cast<long long>(ms) * kMemberCap;
    for (unsigned i = threadIdx.x; i < cnt; i += NT)
      if (sh.mbase + i < static_cast<unsigned>(kMemberCap)) mem[sh.mbase + i] = loc[i];
  }
}

// Among members [0, nm) (keys, exact weights), those in cells [c0, c1] in key
// order: the first at which base + running weight reaches t (> base).  Sets
// sh.r_found, r_key, r_cum (running weight through it) and r_rank (its rank
// among the members of [c0, c1]).  Members are binned by x into kSubBins
// sub-bins (monotone in key order) whose weights are scanned; only the target
// sub-bin's members are sorted (one warp, at most 32); a crowded sub-bin
// (ties) sorts every member of the range instead.
__device__ __noinline__ void resolve(const unsigned long long* mkey, const double* mw, int nm, int c0, int c1,
                                     double base, double t, double temp_d, double* sbm, unsigned* sbc,
                                     unsigned long long* buf, Shared& sh) {
  const Grid g = sh.g;
  const float xtop = static_cast<float>(-ldexp(static_cast<double>(c0) - 0.5, -g.K));  // upper edge of c0
  const float scale = static_cast<float>(ldexp(static_cast<double>(kSubBins), g.K) / (c1 - c0 + 1));
  auto sub_of = [&](unsigned long long k) -> int {  // -1: not in [c0, c1]
    float d, tt;
    const float xh = xof(dval(k), g, &d);
    const int c = cell_of(xh, g, &tt);
    if (c < c0 || c > c1) return -1;
    const float uu = __fmul_rn(__fsub_rn(xtop, xh), scale);  // monotone in -x
    return min(kSubBins - 1, max(0, static_cast<int>(uu)));
  };
  sbm[threadIdx.x] = 0.0;
  sbc[threadIdx.x] = 0u;
  __syncthreads();
  for (int i = threadIdx.x; i < nm; i += NT) {
    const int b = sub_of(mkey[i]);
    if (b < 0) continue;
    atomicAdd(&sbc[b], 1u);
    atomicAdd(&sbm[b], mw[i]);
  }
  __syncthreads();
  const double m = sbm[threadIdx.x];
  const unsigned c = sbc[threadIdx.x];
  double wpre, wtot;
  unsigned cpre, ctot;
  bscan(m, c, sh, &wpre, &cpre, &wtot, &ctot);
  if (threadIdx.x == 0) sh.sb = -1;
  __syncthreads();
  const double before = base + wpre;
  if (c > 0 && before < t && t <= before + m) {
    sh.sb = threadIdx.x;
    sh.sb_base = before;
    sh.sb_n = c;
    sh.sb_cnt_before = cpre;
  }
  __syncthreads();
  const int sb = sh.sb;
  if (sb < 0) {
    if (threadIdx.x == 0) sh.r_found = 0;
    __syncthreads();
    return;
  }
  const int lane = threadIdx.x & 31;
  if (sh.sb_n <= 32u) {
    if (threadIdx.x == 0) sh.nmem = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < nm; i += NT)
      if (sub_of(mkey[i]) == sb) {
        const unsigned q = atomicAdd(&sh.nmem, 1u);
        if (q < 32u) buf[q] = static_cast<unsigned long long>(i);
      }
    __syncthreads();
    if (threadIdx.x < 32) {
      const int cnt = static_cast<int>(min(sh.nmem, 32u));
      const bool have = lane < cnt;
      unsigned long long k = have ? mkey[buf[lane]] : kNoKey;
      double w = have ? mw[buf[lane]] : 0.0;
#pragma unroll
      for (int kk = 2; kk <= 32; kk <<= 1) {
#pragma unroll
        for (int j = kk >> 1; j > 0; j >>= 1) {  // ascending bitonic sort by key, weight alongside
          const unsigned long long pk = __shfl_xor_sync(0xffffffffu, k, j);
          const double pw = __shfl_xor_sync(0xffffffffu, w, j);
          const bool take_min = ((lane & j) == 0) == ((lane & kk) == 0);
          if (take_min ? (pk < k) : (pk > k)) {
            k = pk;
            w = pw;
          }
        }
      }
      double inc = w;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += y;
      }
      const unsigned hits = __ballot_sync(0xffffffffu, have && sh.sb_base + inc >= t);
      const int L = hits ? __ffs(hits) - 1 : 0;
      const unsigned long long kL = __shfl_sync(0xffffffffu, k, L);
      const double iL = __shfl_sync(0xffffffffu, inc, L);
      if (lane == 0) {
        sh.r_found = hits != 0 && sh.nmem <= 32u;
        sh.r_key = kL;
        sh.r_cum = sh.sb_base + iL;
        sh.r_rank = sh.sb_cnt_before + static_cast<unsigned>(L);
      }
    }
    __syncthreads();
    return;
  }
  // crowded sub-bin (ties): sort every member of [c0, c1] by key and walk them
  if (threadIdx.x == 0) sh.nmem = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < nm; i += NT)
    if (sub_of(mkey[i]) >= 0) buf[atomicAdd(&sh.nmem, 1u)] = mkey[i];
  __syncthreads();
  const int cnt = static_cast<int>(sh.nmem);
  const int P = next_pow2(max(cnt, 2));
  for (int i = cnt + threadIdx.x; i < P; i += NT) buf[i] = kNoKey;
  __syncthreads();
  bitonic_sort_u64(reinterpret_cast<uint64_t*>(buf), P);
  if (threadIdx.x == 0) {
    double cm = base;
    int hit = -1;
    for (int i = 0; i < cnt; ++i) {
      cm += ref_weight(dval(buf[i]), g.M, temp_d);
      if (cm >= t) {
        hit = i;
        break;
      }
    }
    sh.r_found = hit >= 0;
    if (hit >= 0) {
      sh.r_key = buf[hit];
      sh.r_cum = cm;
      sh.r_rank = static_cast<unsigned>(hit);
    }
  }
  __syncthreads();
}

// The row's pick among the gathered members: the top-p cutoff, then the draw
// within the kept prefix; results stored, or the row listed for the staged
// kernel.
__device__ __noinline__ void merge_c(int row, unsigned char* smem, Shared& sh) {
  const NucArgs& p = sh.p;
  const DevOpts& o = sh.o;
  const RowArgs& a = p.a;
  const int ms = row % kChunkRows;
  const Targets* tg = p.tg + ms;
  if (threadIdx.x == 0) sh.g = row_grid(p.rs + row, o.temp);
  __syncthreads();
  const Grid g = sh.g;
  unsigned long long* mkey = reinterpret_cast<unsigned long long*>(smem);
  double* mw = reinterpret_cast<double*>(mkey + kMemberCap);
  unsigned long long* buf = reinterpret_cast<unsigned long long*>(mw + kMemberCap);
  double* sbm = reinterpret_cast<double*>(buf + kMemberCap);
  unsigned* sbc = reinterpret_cast<unsigned*>(sbm + kSubBins);
  bool ok = __ldcg(&tg->fail) == 0;
  const unsigned nmem = __ldcg(&tg->nmem);
  if (nmem > static_cast<unsigned>(kMemberCap)) ok = false;
  const int nm = static_cast<int>(min(nmem, static_cast<unsigned>(kMemberCap)));
  const double temp_d = static_cast<double>(o.temp);
  if (ok) {
    const unsigned long long* mem = p.members + static_cast<long long>(ms) * kMemberCap;
    for (int i = threadIdx.x; i < nm; i += NT) {
      const unsigned long long k = __ldcg(mem + i);
      mkey[i] = k;
      mw[i] = ref_weight(dval(k), g.M, temp_d);
    }
  }
  __syncthreads();
  double tot = 0.0;
  unsigned keep = static_cast<unsigned>(o.k);
  int out_id = 0;
  if (ok) {
    const int use_p = __ldcg(&tg->use_p);
    const int A0 = __ldcg(&tg->A0), A1 = __ldcg(&tg->A1), B0 = __ldcg(&tg->B0), B1 = __ldcg(&tg->B1);
    const double S = __ldcg(&tg->S), u = __ldcg(&tg->u);
    tot = S;
    unsigned long long cut_key = kNoKey;
    if (use_p) {  // the cutoff: first member at which the running mass reaches top_p * S
      resolve(mkey, mw, nm, A0, A1, __ldcg(&tg->cut_base), __ldcg(&tg->tp), temp_d, sbm, sbc, buf, sh);
      ok = sh.r_found != 0;
      tot = sh.r_cum;
      keep = __ldcg(&tg->cut_before) + sh.r_rank + 1u;
      cut_key = sh.r_key;
    }
    const int use_m = __ldcg(&tg->use_m);
    if (ok && use_m == 1 && __ldcg(&tg->q_over) != 0u) ok = false;
    if (ok && use_m == 1) {
      // min-p (src/sampler.cpp:86-91): the columns with weight >= min_p (the
      // max's weight is exp(0) = 1), at least the first; the kept prefix is
      // the shorter of the two cuts
      unsigned km = __ldcg(&tg->q_before) + __ldcg(&tg->q_n);
      double tm = __ldcg(&tg->q_base) + ldexp(static_cast<double>(__ldcg(&tg->q_mass)), -kQFix);
      unsigned long long lastm = __ldcg(&tg->q_n) ? __ldcg(&tg->q_last) : kNoKey;
      if (km == 0u) {  // min_p above every weight: the first column alone, weight exp(0) = 1
        km = 1u;
        lastm = __ldcg(&tg->q_first);
        tm = 1.0;
        if (lastm == kNoKey) ok = false;
      }
      if (km < keep) {
        keep = km;
        tot = tm;
        cut_key = lastm;
      }
    } else if (ok && use_m == 2) {  // min-p keeps every cell
      const unsigned km = __ldcg(&tg->q_before);
      if (km < keep) {
        keep = km;
        tot = __ldcg(&tg->q_base);
      }
    }
    if (ok) {  // the draw: first kept member at which the running mass reaches u * tot
      const double r = u * tot;
      const double t = r > 0.0 ? r : 4.9406564584124654e-324;
      const double draw_base = __ldcg(&tg->draw_base);
      if (!(t > draw_base)) {
        ok = false;
      } else {
        resolve(mkey, mw, nm, B0, B1, draw_base, t, temp_d, sbm, sbc, buf, sh);
        ok = sh.r_found != 0 && sh.r_key <= cut_key;
        out_id = static_cast<int>(did(sh.r_key));
      }
    }
  }
  if (threadIdx.x == 0) {
    if (!ok) {
      to_fallback(p, row);
    } else {
      if (a.rng) {
        a.rng[2ll * row] = __ldcg(&tg->s1);
        a.rng[2ll * row + 1] = __ldcg(&tg->s0);
      }
      a.out_ids[row] = out_id;
      ring_append(a, row, out_id);
      if (a.stats) {
        const double nan = __longlong_as_double(0x7ff8000000000000ll);
        write_stats(a.stats + row, __ldcg(&tg->S), tot, __ldcg(&tg->u), nan, nan, o.k, static_cast<int>(keep),
                    out_id, 0);
      }
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------- kernels ----
// One CTA per (row, slice): blockIdx.x = (row - row0) * ns + slice.
__device__ __forceinline__ void setup(const NucArgs& p, const DevOpts& o, Shared& sh) {
  if (threadIdx.x == 0) {
    sh.p = p;
    sh.o = o;
  }
  __syncthreads();
}

// One kernel per pass, each with the resources its pass needs: the A pass
// streams with no shared memory at 8 CTAs per SM, the B pass keeps its
// histogram (and the row merge of its last slice) in 24 KB, the C pass its
// members in 16 KB; the resolve runs one CTA per row.  CTA i of the A, B and C
// kernels takes row first + i / ns, slice i mod ns.
__global__ void __launch_bounds__(NT, 8) nuc_a_kernel(const NucArgs p, const DevOpts o) {
  __shared__ Shared sh;
  const int j = static_cast<int>(blockIdx.x);
  setup(p, o, sh);
  run_a(p.rowa + j / p.ns, j % p.ns, sh);
}
__global__ void __launch_bounds__(NT, kBBlocks) nuc_b_kernel(const NucArgs p, const DevOpts o) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ Shared sh;
  const int j = static_cast<int>(blockIdx.x);
  setup(p, o, sh);
  run_b(p.rowb + j / p.ns, j % p.ns, smem, sh);
}
template <bool kMinP>
__global__ void __launch_bounds__(NT, kCBlocks) nuc_c_kernel(const NucArgs p, const DevOpts o) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ Shared sh;
  const int j = static_cast<int>(blockIdx.x);
  setup(p, o, sh);
  run_c<kMinP>(p.rowc + j / p.ns, j % p.ns, smem, sh);
}
__global__ void __launch_bounds__(NT, 4) nuc_r_kernel(const NucArgs p, const DevOpts o) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ Shared sh;
  setup(p, o, sh);
  merge_c(p.rowc + static_cast<int>(blockIdx.x), smem, sh);
}

}  // namespace nuc

// ------------------------------------------------------------- launcher ---
bool nucleus_eligible(const DevOpts& o, int vocab) {
  return !o.greedy && o.k >= vocab && !o.penalize && vocab >= kNucleusMinVocab;
}

static int slices_of(int ncols) { return (ncols + nuc::kSliceCols - 1) / nuc::kSliceCols; }

size_t nucleus_scratch_bytes(int rows, int ncols) { return nuc::layout(rows, slices_of(ncols)).bytes; }

cudaError_t launch_nucleus(const RowArgs& a, const DevOpts& o, void* scratch, cudaStream_t s) {
  using namespace nuc;
  const int ns = slices_of(a.ncols);
  const Layout l = layout(a.rows, ns);
  char* b = static_cast<char*>(scratch);
  cudaError_t e = cudaMemsetAsync(b, 0, l.zero_bytes, s);
  if (e != cudaSuccess) return e;
  NucArgs p;
  p.a = a;
  p.ns = ns;
  p.slice = (((a.ncols + ns - 1) / ns) + 3) & ~3;
  p.fb_count = reinterpret_cast<unsigned*>(b);
  p.rs = reinterpret_cast<RowState*>(b + l.off_rs);
  p.fb_list = reinterpret_cast<int*>(b + l.off_fb);
  p.sums = reinterpret_cast<SliceSum*>(b + l.off_sum);
  p.cells = reinterpret_cast<uint2*>(b + l.off_cells);
  p.tg = reinterpret_cast<Targets*>(b + l.off_tg);
  p.members = reinterpret_cast<unsigned long long*>(b + l.off_mem);
  // the resolve's shared memory is above the 48 KB default (per device)
  static unsigned long long attrs = 0;
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 64 || !(attrs >> dev & 1ull)) {
    e = cudaFuncSetAttribute(nuc_r_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kRSmem));
    if (e != cudaSuccess) return e;
    if (dev < 64) attrs |= 1ull << dev;
  }
  for (int r0 = 0; r0 < a.rows; r0 += kChunkRows) {
    const int n = std::min(kChunkRows, a.rows - r0);
    p.rowa = p.rowb = p.rowc = r0;
    p.na = p.nb = p.nc = n;
    nuc_a_kernel<<<n * ns, NT, 0, s>>>(p, o);
    nuc_b_kernel<<<n * ns, NT, kBSmem, s>>>(p, o);
    if (o.min_p > 0.0f)
      nuc_c_kernel<true><<<n * ns, NT, kCSmem, s>>>(p, o);
    else
      nuc_c_kernel<false><<<n * ns, NT, kCSmem, s>>>(p, o);
    nuc_r_kernel<<<n, NT, kRSmem, s>>>(p, o);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // the rows it could not settle, on the staged cluster kernel
  return launch_general_list(a, o, p.fb_list, p.fb_count, a.rows, s);
}

cudaError_t nucleus_fallbacks(const void* scratch, cudaStream_t s, unsigned* out) {
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return e;
  unsigned c = 0;
  e = cudaMemcpy(&c, scratch, sizeof(c), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) *out = c;
  return e;
}

cudaError_t read_nucleus_status(unsigned* st, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(st, nuc::g_nuc_status, sizeof(unsigned));
  if (e != cudaSuccess) return e;
  if (clear && *st) {
    const unsigned z = 0;
    e = cudaMemcpyToSymbol(nuc::g_nuc_status, &z, sizeof(unsigned));
  }
  return e;
}

}  // namespace vb
