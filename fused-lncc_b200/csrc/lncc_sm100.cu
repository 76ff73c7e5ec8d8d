// liblncc_sm100: fused 3-D LNCC loss + dL/dpred for B200 (sm_100a).
//
// One kernel launch reads pred and target once and produces both the cc partial sums and the
// gradient. The reference needs two kernels, four fp32 maps and two torch ops for the same result:
// lncc_fwd (fused_lncc/csrc/lncc3d.cu:25-110), lncc_bwd (lncc3d.cu:166-235), `ncc.mean()` and
// `* (-grad_out/M)` (fused_lncc/__init__.py:62,73).
//
// Sweep design (lncc_sweep_kernel). A thread block owns a TH x TW tile of output columns (H, W) of one
// volume and walks along D through a chunk of output planes. Per input plane j it runs:
//   A  D-pass   : running sums along D of p, t, p*p, t*t, p*t at every footprint column
//                 ((TH+4r) x (TW+4r)), using a k-deep ring of raw planes in shared memory;
//   B  H-pass   : box along H of those five fields        -> (TH+2r) x (TW+4r)
//   C  W-pass   : box along W -> the five k^3 window sums at stat plane j-r on (TH+2r) x (TW+2r),
//                 then cc (summed into the block's loss partial) and the three adjoint fields;
//   D  H-pass   : box along H of the adjoints             -> TH x (TW+2r)
//   E  W-pass + D running sum (k-deep ring of boxed adjoint planes) -> the adjoint box at output
//                 plane j-2r on TH x TW, combined with p, t into dL/dpred.
// Nothing but the gradient and one fp64 partial per block reaches global memory.
//
// Statistics are kept multiplied by n = k^3, so that constant inputs cancel exactly as with the
// reference's division by n (lncc3d.cu:93-97):
//   X = n*Spt - Sp*St = n*cross,  VP = max(n*Spp - Sp^2, 0) + n*dr = n*var_p,  VT likewise,
//   cc = X^2/(VP*VT).  With w = X/(VP*VT) the adjoints of lncc3d.cu:101-104 are
//   Cc = 2n*c, Bc = -n*b, A = -2*a  for  c = w, b = w*w*VT, a = w*(St - w*VT*Sp),
// and d(sum cc)/dp = box(A) + 2p*box(Bc) + t*box(Cc) = 2*(n*t*box(c) - n*p*box(b) - box(a)).
#include "lncc.h"
#include "lncc_check.cuh"

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdlib.h>
#include <atomic>
#include <mutex>

#define LNCC_VERSION_NUM 100  // 0.1.0

#include "lncc_compat.cuh"
#include "lncc_ws.cuh"

namespace lncc {

// ------------------------------------------------------------------------------------------------
// element access
// ------------------------------------------------------------------------------------------------
template <typename S> __device__ __forceinline__ float ldf(const S* p);
template <> __device__ __forceinline__ float ldf<float>(const float* p) { return __ldg(p); }
template <> __device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(__ldg(p));
}
template <typename S> __device__ __forceinline__ void stg(S* p, float v);
template <> __device__ __forceinline__ void stg<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void stg<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ float ldf<__half>(const __half* p) { return __half2float(__ldg(p)); }
__device__ __forceinline__ float tof(float v) { return v; }
__device__ __forceinline__ float tof(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float tof(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ void stg<__half>(__half* p, float v) { *p = __float2half_rn(v); }

// ------------------------------------------------------------------------------------------------
// geometry of the sweep kernel (all in fp32 words of shared memory)
// ------------------------------------------------------------------------------------------------
template <int R, int TH, int TW, int NT>
struct SweepCfg {
  static constexpr int K = 2 * R + 1;
  static constexpr int W0 = TW + 4 * R, H0 = TH + 4 * R, F0 = W0 * H0;  // raw footprint
  static constexpr int W1 = TW + 2 * R, H1 = TH + 2 * R, F1 = W1 * H1;  // stat positions
  static constexpr int F2 = TH * TW;                                    // outputs
  static constexpr int PPT = (F0 + NT - 1) / NT;                        // footprint columns per thread
  static constexpr int OFF_RING = 0;                        // [K][2][F0] raw p, t planes
  static constexpr int OFF_DS = OFF_RING + K * 2 * F0;      // [5][F0]    D-window sums
  static constexpr int OFF_HS = OFF_DS + 5 * F0;            // [5][H1][W0] after the H box
  static constexpr int OFF_ADJ = OFF_HS + 5 * H1 * W0;      // [3][H1][W1] adjoints at stat plane
  static constexpr int OFF_AH = OFF_ADJ + 3 * F1;           // [3][TH][W1] adjoints after H box
  static constexpr int OFF_RING2 = OFF_AH + 3 * TH * W1;    // [K][3][F2] HW-boxed adjoint planes
  static constexpr int OFF_RED = (OFF_RING2 + K * 3 * F2 + 3) & ~3;  // NT/32 doubles
  static constexpr int NWORDS = OFF_RED + 2 * (NT / 32);
  static constexpr size_t SMEM_BYTES = size_t(NWORDS) * 4;
  // W-pass (phase C) run length: largest of 4,3,2,1 dividing W1
  static constexpr int M1 = (W1 % 4 == 0) ? 4 : (W1 % 3 == 0) ? 3 : (W1 % 2 == 0) ? 2 : 1;
  static_assert(F2 <= NT * 2, "phase E maps at most two outputs per thread");
};

struct SweepArgs {
  const void* p;
  const void* t;
  void* g;
  double* partials;
  const float* gscale_dev;
  float gscale;  // multiplies d(sum cc)/dp
  float n;       // k^3
  float dr;
  int D, H, W;
  int z_begin, z_end, dchunk;
  int tiles_w, tiles_h, nchunks;
  unsigned* abort_word;  // workspace word that lncc_check_abort reads; this kernel never waits, so it only clears it
  int64_t n_in, n_g, n_parts;  // elements of p / t, of g, and partials (range checks of the checked build)
};

template <int R, int TH, int TW, int NT, typename S, bool GRAD>
__global__ void __launch_bounds__(NT) lncc_sweep_kernel(const SweepArgs a) {
  using C = SweepCfg<R, TH, TW, NT>;
  constexpr int K = C::K, W0 = C::W0, F0 = C::F0, W1 = C::W1, H1 = C::H1, F1 = C::F1, F2 = C::F2;
  constexpr int PPT = C::PPT;
  extern __shared__ __align__(16) float sm[];
  float* ring = sm + C::OFF_RING;
  float* DS = sm + C::OFF_DS;
  float* HS = sm + C::OFF_HS;
  float* ADJ = sm + C::OFF_ADJ;
  float* AH = sm + C::OFF_AH;
  float* ring2 = sm + C::OFF_RING2;
  double* red = reinterpret_cast<double*>(sm + C::OFF_RED);

  const int tid = threadIdx.x;
  int bid = blockIdx.x;
  const int tw = bid % a.tiles_w;
  bid /= a.tiles_w;
  const int th = bid % a.tiles_h;
  bid /= a.tiles_h;
  const int ch = bid % a.nchunks;
  const int64_t b = bid / a.nchunks;
  const int x0 = tw * TW, y0 = th * TH;
  const int zs = a.z_begin + ch * a.dchunk;
  const int ze = min(zs + a.dchunk, a.z_end);
  const int D = a.D, H = a.H, W = a.W;
  if (a.abort_word && tid == 0 && blockIdx.x == 0) *a.abort_word = 0u;
  const int64_t HW = int64_t(H) * W;
  const S* __restrict__ P = reinterpret_cast<const S*>(a.p) + b * D * HW;
  const S* __restrict__ T = reinterpret_cast<const S*>(a.t) + b * D * HW;
  S* __restrict__ G = nullptr;
  if (GRAD) G = reinterpret_cast<S*>(a.g) + b * int64_t(a.z_end - a.z_begin) * HW;
  const float nf = a.n, ndr = a.n * a.dr;
  float gs = 0.f;
  if (GRAD) gs = 2.f * a.gscale * (a.gscale_dev ? __ldg(a.gscale_dev) : 1.f);

  for (int i = tid; i < K * 2 * F0; i += NT) ring[i] = 0.f;
  if (GRAD)
    for (int i = tid; i < K * 3 * F2; i += NT) ring2[i] = 0.f;

  // phase A ownership: footprint column q = tid + i*NT
  int aoff[PPT];
  bool aval[PPT];
#pragma unroll
  for (int i = 0; i < PPT; ++i) {
    const int q = tid + i * NT;
    const int r0 = q / W0, c0 = q % W0;
    const int gy = y0 - 2 * R + r0, gx = x0 - 2 * R + c0;
    aval[i] = (q < F0) && gy >= 0 && gy < H && gx >= 0 && gx < W;
    aoff[i] = aval[i] ? gy * W + gx : 0;
  }
  float s5[PPT][5];
  float np_[PPT], nt_[PPT];
#pragma unroll
  for (int i = 0; i < PPT; ++i) {
#pragma unroll
    for (int f = 0; f < 5; ++f) s5[i][f] = 0.f;
  }
  const int j0 = zs - 2 * R, j1 = ze + 2 * R;
  auto load_plane = [&](int j) {
    const bool pv = (j >= 0) && (j < D);
#pragma unroll
    for (int i = 0; i < PPT; ++i) {
      np_[i] = 0.f;
      nt_[i] = 0.f;
      if (pv && aval[i] && LNCC_IN(b * D * HW + int64_t(j) * HW + aoff[i], 1, a.n_in)) {
        np_[i] = ldf<S>(P + int64_t(j) * HW + aoff[i]);
        nt_[i] = ldf<S>(T + int64_t(j) * HW + aoff[i]);
      }
    }
  };
  load_plane(j0);

  // phase E ownership (one or two outputs per thread)
  constexpr int E_PER = (F2 + NT - 1) / NT;
  float T3[E_PER][3];
#pragma unroll
  for (int e = 0; e < E_PER; ++e) T3[e][0] = T3[e][1] = T3[e][2] = 0.f;

  float acc = 0.f;  // this thread's share of sum(cc)
  __syncthreads();

  for (int j = j0, it = 0; j < j1; ++j, ++it) {
    const int slot = it % K;
    // ---- A: D running sums at every footprint column --------------------------------------------
#pragma unroll
    for (int i = 0; i < PPT; ++i) {
      const int q = tid + i * NT;
      if (q < F0) {
        const float op = ring[(slot * 2 + 0) * F0 + q];
        const float ot = ring[(slot * 2 + 1) * F0 + q];
        const float p = np_[i], t = nt_[i];
        s5[i][0] += p - op;
        s5[i][1] += t - ot;
        s5[i][2] = fmaf(p, p, fmaf(-op, op, s5[i][2]));
        s5[i][3] = fmaf(t, t, fmaf(-ot, ot, s5[i][3]));
        s5[i][4] = fmaf(p, t, fmaf(-op, ot, s5[i][4]));
        if (LNCC_IN((slot * 2 + 1) * F0 + q, 1, K * 2 * F0)) {
          ring[(slot * 2 + 0) * F0 + q] = p;
          ring[(slot * 2 + 1) * F0 + q] = t;
        }
#pragma unroll
        for (int f = 0; f < 5; ++f)
          if (LNCC_IN(f * F0 + q, 1, 5 * F0)) DS[f * F0 + q] = s5[i][f];
      }
    }
    if (j + 1 < j1) load_plane(j + 1);
    if (j < zs) {  // warm-up: the D sums are not complete yet
      __syncthreads();
      continue;
    }
    __syncthreads();
    const int c1 = j - R;  // stat plane produced in this step
    const bool c1_in = (c1 >= 0) && (c1 < D);
    // ---- B: H box of the five D sums: (H1 x W0) ---------------------------------------------------
    if (c1_in) {
      for (int task = tid; task < 5 * W0; task += NT) {
        const int f = task / W0, c = task % W0;
        const float* src = DS + f * F0 + c;
        float* dst = HS + f * H1 * W0 + c;
        float s = 0.f;
#pragma unroll
        for (int d = 0; d < 2 * R + 1; ++d) s += src[d * W0];
        if (LNCC_IN(f * H1 * W0 + c, 1, 5 * H1 * W0)) dst[0] = s;
        for (int r = 1; r < H1; ++r) {
          if (!LNCC_IN(f * F0 + (r + 2 * R) * W0 + c, 1, 5 * F0)) break;
          s += src[(r + 2 * R) * W0] - src[(r - 1) * W0];
          if (LNCC_IN(f * H1 * W0 + r * W0 + c, 1, 5 * H1 * W0)) dst[r * W0] = s;
        }
      }
    }
    __syncthreads();
    // ---- C: W box -> window sums -> cc, adjoints at the stat plane ---------------------------------
    {
      constexpr int M1 = C::M1, NSEG = W1 / M1;
      const bool c1_own = c1_in && (c1 >= zs) && (c1 < ze);
      for (int task = tid; c1_in && task < H1 * NSEG; task += NT) {
        const int r = task / NSEG, cs = (task % NSEG) * M1;
        float st5[5][M1];
#pragma unroll
        for (int f = 0; f < 5; ++f) {
          const float* src = HS + f * H1 * W0 + r * W0 + cs;
          float s = 0.f;
#pragma unroll
          for (int d = 0; d < 2 * R + 1; ++d) s += src[d];
          st5[f][0] = s;
#pragma unroll
          for (int m = 1; m < M1; ++m) {
            s += src[m + 2 * R] - src[m - 1];
            st5[f][m] = s;
          }
        }
        const int gy = y0 - R + r;
        const bool row_in = c1_in && gy >= 0 && gy < H;
        const bool row_own = c1_own && (r >= R) && (r < R + TH) && (gy < H);
#pragma unroll
        for (int m = 0; m < M1; ++m) {
          const int c = cs + m;
          const int gx = x0 - R + c;
          const bool in = row_in && gx >= 0 && gx < W;
          const float Sp = st5[0][m], St = st5[1][m], Spp = st5[2][m], Stt = st5[3][m], Spt = st5[4][m];
          const float X = fmaf(nf, Spt, -(Sp * St));
          const float VP = fmaxf(fmaf(nf, Spp, -(Sp * Sp)), 0.f) + ndr;
          const float VT = fmaxf(fmaf(nf, Stt, -(St * St)), 0.f) + ndr;
          const float w = X * __frcp_rn(VP * VT);
          const float cc = X * w;
          if (in && row_own && c >= R && c < R + TW && gx < W) acc += (cc >= 1.f) ? 1.f : cc;
          if (GRAD) {
            const bool live = in && (cc < 1.f);  // NaN and cc >= 1 give zero adjoints (lncc3d.cu:100-107)
            const float wv = w * VT;
            const float bq = w * wv;
            const float aq = w * fmaf(-wv, Sp, St);
            if (LNCC_IN(2 * F1 + r * W1 + c, 1, 3 * F1) && LNCC_IN(r * W1 + c, 1, F1)) {
              ADJ[0 * F1 + r * W1 + c] = live ? aq : 0.f;
              ADJ[1 * F1 + r * W1 + c] = live ? bq : 0.f;
              ADJ[2 * F1 + r * W1 + c] = live ? w : 0.f;
            }
          }
        }
      }
      if (GRAD && !c1_in) {
        for (int i = tid; i < 3 * F1; i += NT) ADJ[i] = 0.f;
      }
    }
    if (!GRAD) {
      __syncthreads();
      continue;
    }
    __syncthreads();
    // ---- D: H box of the adjoints: (TH x W1) ------------------------------------------------------
    {
      constexpr int SEGH = (TH % 2 == 0) ? 2 : 1, LH = TH / SEGH;
      for (int task = tid; task < 3 * W1 * SEGH; task += NT) {
        const int f = task / (W1 * SEGH), rem = task % (W1 * SEGH);
        const int c = rem % W1, r0 = (rem / W1) * LH;
        const float* src = ADJ + f * F1 + c;
        float* dst = AH + f * TH * W1 + c;
        float s = 0.f;
#pragma unroll
        for (int d = 0; d < 2 * R + 1; ++d) s += src[(r0 + d) * W1];
        if (LNCC_IN(f * TH * W1 + r0 * W1 + c, 1, 3 * TH * W1)) dst[r0 * W1] = s;
#pragma unroll
        for (int r = r0 + 1; r < r0 + LH; ++r) {
          s += src[(r + 2 * R) * W1] - src[(r - 1) * W1];
          if (LNCC_IN(f * F1 + (r + 2 * R) * W1 + c, 1, 3 * F1) && LNCC_IN(f * TH * W1 + r * W1 + c, 1, 3 * TH * W1))
            dst[r * W1] = s;
        }
      }
    }
    __syncthreads();
    // ---- E: W box, D running sum, combine ----------------------------------------------------------
    {
      const int slot2 = it % K;       // ring2 slot of stat plane c1 (and of c1 - K)
      const int pslot = (it + 1) % K;  // raw slot of output plane j - 2R
      const int c2 = j - 2 * R;
      const bool c2_out = (c2 >= zs) && (c2 < ze);
#pragma unroll
      for (int e = 0; e < E_PER; ++e) {
        const int q = tid + e * NT;
        if (q < F2) {
          const int r = q / TW, c = q % TW;
          float v[3];
#pragma unroll
          for (int f = 0; f < 3; ++f) {
            const float* src = AH + f * TH * W1 + r * W1 + c;
            float s = 0.f;
#pragma unroll
            for (int d = 0; d < 2 * R + 1; ++d) s += src[d];
            v[f] = s;
            float* rs = ring2 + (slot2 * 3 + f) * F2 + q;
            if (LNCC_IN((slot2 * 3 + f) * F2 + q, 1, K * 3 * F2)) {
              T3[e][f] += s - *rs;
              *rs = s;
            }
          }
          const int gy = y0 + r, gx = x0 + c;
          if (c2_out && gy < H && gx < W) {
            const int q0 = (r + 2 * R) * W0 + (c + 2 * R);
            const float p = ring[(pslot * 2 + 0) * F0 + q0];
            const float t = ring[(pslot * 2 + 1) * F0 + q0];
            const float gval = gs * fmaf(nf, fmaf(t, T3[e][2], -p * T3[e][1]), -T3[e][0]);
            if (LNCC_IN(b * int64_t(a.z_end - a.z_begin) * HW + int64_t(c2 - a.z_begin) * HW + gy * W + gx, 1, a.n_g) &&
                LNCC_IN((pslot * 2 + 1) * F0 + q0, 1, K * 2 * F0))
              stg<S>(G + int64_t(c2 - a.z_begin) * HW + gy * W + gx, gval);
          }
        }
      }
    }
    __syncthreads();
  }

  // ---- block partial of sum(cc), fixed order ---------------------------------------------------------
  double dacc = acc;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dacc += __shfl_down_sync(0xffffffffu, dacc, o);
  if ((tid & 31) == 0) red[tid >> 5] = dacc;
  __syncthreads();
  if (tid == 0) {
    double s = 0.0;
    for (int w = 0; w < NT / 32; ++w) s += red[w];
    if (LNCC_IN(blockIdx.x, 1, a.n_parts)) a.partials[blockIdx.x] = s;
  }
}

// Deterministic second pass: one block sums the per-block partials in a fixed order.
__global__ void __launch_bounds__(1024) lncc_reduce_kernel(const double* __restrict__ partials, int n,
                                                           double* sum_out, float* loss_out,
                                                           double count) {
  __shared__ double sh[32];
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += partials[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double tot = 0.0;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) tot += sh[w];
    if (sum_out) *sum_out = tot;
    if (loss_out) *loss_out = float(1.0 - tot / count);
  }
}

// Loss of a batch sharded over ranks, one GPU each (lncc_peer_loss). Lane l (< world) writes this
// rank's sum, then the epoch with system-scope release, into slot `rank` of rank l's exchange buffer
// (peer memory over NVLink), then waits, bounded, until slot l of this rank's own buffer carries the
// epoch and reads rank l's sum; the sums are added in rank order, so every rank gets the same bits.
// Buffers: [2 epoch parities][world writers] x {double sum, uint64 epoch}; a rank one step ahead writes
// the other parity, and two steps ahead it cannot be, since its next step needs this rank's sum.
__global__ void __launch_bounds__(32) lncc_peer_loss_kernel(const double* __restrict__ local_sum,
                                                          uint64_t* const* __restrict__ slots, int rank, int world,
                                                          uint64_t epoch, double count, double* sum_out,
                                                          float* loss_out, unsigned* abort_word,
                                                          unsigned long long limit_ns) {
  const int l = threadIdx.x;
  const int par = int(epoch & 1u);
  const double v = *local_sum;
  if (l < world) {
    uint64_t* dst = slots[l] + 2 * (par * world + rank);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(static_cast<uint64_t>(__double_as_longlong(v)))
                 : "memory");
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(dst + 1), "l"(epoch) : "memory");
  }
  double got = 0.0;
  bool ok = true;
  if (l < world) {
    const uint64_t* src = slots[rank] + 2 * (par * world + l);
    unsigned long long t0 = 0, t = 0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (;;) {
      uint64_t e;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(e) : "l"(src + 1) : "memory");
      if (e == epoch) break;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > limit_ns) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
    if (ok) {
      uint64_t bits;
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(bits) : "l"(src) : "memory");
      got = __longlong_as_double(static_cast<long long>(bits));
    }
  }
  double tot = 0.0;
  for (int r = 0; r < world; ++r) tot += __shfl_sync(0xffffffffu, got, r);
  const bool all_ok = __all_sync(0xffffffffu, ok);
  if (l == 0) {
    if (!all_ok) {
      tot = __longlong_as_double(0x7ff8000000000000ll);
      if (abort_word) atomicOr(abort_word, 1u);
    }
    if (sum_out) *sum_out = tot;
    if (loss_out) *loss_out = float(1.0 - tot / count);
  }
}

template <typename S>
__global__ void lncc_scale_grad_kernel(S* __restrict__ g, int64_t n, const float* __restrict__ go) {
  const float s = __ldg(go);
  if (s == 1.f) return;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    stg<S>(g + i, tof(g[i]) * s);  // a plain load: g is written by this kernel
  }
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------
constexpr int kTH = 16, kTW = 16, kNT = 256;

struct Plan {
  int R;
  int tiles_w, tiles_h, nchunks, dchunk;
  int64_t nblocks;
};

static int sm_count_current() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if (cache[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev] = v;
  }
  return cache[dev];
}

static Plan make_plan(int64_t B, int64_t H, int64_t W, int k, int64_t z_begin, int64_t z_end) {
  Plan pl;
  pl.R = k / 2;
  pl.tiles_w = int((W + kTW - 1) / kTW);
  pl.tiles_h = int((H + kTH - 1) / kTH);
  const int64_t nout = z_end - z_begin;
  const int64_t base = B * pl.tiles_w * pl.tiles_h;
  const int64_t target = 4LL * sm_count_current();
  int64_t nch = 1;
  if (base < target) nch = (target + base - 1) / base;
  const int64_t min_chunk = 16;
  int64_t maxch = (nout + min_chunk - 1) / min_chunk;
  if (maxch < 1) maxch = 1;
  if (nch > maxch) nch = maxch;
  int64_t dch = (nout + nch - 1) / nch;
  nch = (nout + dch - 1) / dch;
  pl.nchunks = int(nch);
  pl.dchunk = int(dch);
  pl.nblocks = base * nch;
  return pl;
}

template <int R, typename S, bool GRAD>
static cudaError_t launch_sweep(const SweepArgs& a, int64_t nblocks, cudaStream_t st) {
  using C = SweepCfg<R, kTH, kTW, kNT>;
  auto kfn = lncc_sweep_kernel<R, kTH, kTW, kNT, S, GRAD>;
  // The opt-in shared memory size is a per-device function attribute: set it once per device.
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (!bit || !(done.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(C::SMEM_BYTES));
    if (e != cudaSuccess) return e;
    done.fetch_or(bit, std::memory_order_acq_rel);
  }
  kfn<<<dim3(unsigned(nblocks)), dim3(kNT), C::SMEM_BYTES, st>>>(a);
  return cudaGetLastError();
}

template <typename S, bool GRAD>
static cudaError_t dispatch_r(int R, const SweepArgs& a, int64_t nblocks, cudaStream_t st) {
  switch (R) {
    case 1: return launch_sweep<1, S, GRAD>(a, nblocks, st);
    case 2: return launch_sweep<2, S, GRAD>(a, nblocks, st);
    case 3: return launch_sweep<3, S, GRAD>(a, nblocks, st);
    case 4: return launch_sweep<4, S, GRAD>(a, nblocks, st);
    default: return cudaErrorInvalidValue;
  }
}

static size_t smem_needed(int R) {
  switch (R) {
    case 1: return SweepCfg<1, kTH, kTW, kNT>::SMEM_BYTES;
    case 2: return SweepCfg<2, kTH, kTW, kNT>::SMEM_BYTES;
    case 3: return SweepCfg<3, kTH, kTW, kNT>::SMEM_BYTES;
    case 4: return SweepCfg<4, kTH, kTW, kNT>::SMEM_BYTES;
    default: return 0;
  }
}

static bool valid_k(int k) { return k == 3 || k == 5 || k == 7 || k == 9; }
static bool valid_dtype(int dtype) { return dtype == LNCC_F32 || dtype == LNCC_BF16 || dtype == LNCC_F16; }
static size_t dtype_size(int dtype) { return dtype == LNCC_F32 ? 4 : 2; }
// Calls f with a value of the element type of `dtype` (float, __nv_bfloat16 or __half); the caller
// has checked valid_dtype.
template <typename F>
static auto with_dtype(int dtype, F&& f) {
  if (dtype == LNCC_F32) return f(float{});
  if (dtype == LNCC_BF16) return f(__nv_bfloat16{});
  return f(__half{});
}

// Workspace layout: a 16-byte header whose first word records a timed-out wait of the last call
// (lncc_check_abort), then the fp64 loss partials.
constexpr size_t kWsHeader = 16;

// ------------------------------------------------------------------------------------------------
// process-wide switches
// ------------------------------------------------------------------------------------------------
static std::atomic<int> g_kernel_choice{0};  // 0 auto, 1 sweep, 3 warp-specialised (2: retired)
static std::atomic<int> g_companion{1};      // warp-specialised kernel: companion launch on idle SMs
// set by lncc_fused_forward_noalloc for its call: one launch, so no library stream or events to make
static thread_local bool t_single_launch = false;

// ------------------------------------------------------------------------------------------------
// warp-specialised cluster kernel host side (lncc_ws.cuh)
// ------------------------------------------------------------------------------------------------
constexpr int kWsMaxCluster = 8;   // portable cluster size; taller planes are cut into row tiles
constexpr int kWsMaxTall = 16;     // non-portable cluster size, tried for planes of 129 - 256 rows

// Global-memory chunk width of the kernel for this call: 8 columns (256-bit fp32 / 128-bit bf16
// accesses) when W % 8 == 0 and the base pointers are aligned to a chunk, else 4 columns when
// W % 4 == 0 and aligned to that; 0 = the kernel does not apply.
static int ws_chunk(int64_t W, int dtype, const void* p, const void* t, const void* g) {
  const size_t esz = dtype_size(dtype);
  auto aligned = [&](uintptr_t al) {
    return !((uintptr_t(p) % al) || (uintptr_t(t) % al) || (g && (uintptr_t(g) % al)));
  };
  if (W % 8 == 0 && aligned(8 * esz)) return 8;
  if (W % 4 == 0 && aligned(4 * esz)) return 4;
  return 0;
}

template <int R, typename S, bool GRAD, int CW, bool ASSIST>
static auto ws_kernel_ptr() {
  return ws::lncc_ws_kernel<R, S, GRAD, CW, ASSIST>;
}
template <int R>
static constexpr int ws_smem_r() {
  return ws::smem_bytes<R>();
}

template <int R, typename S, bool GRAD, int CW, bool ASSIST>
static cudaError_t ws_prepare(const void** fn_out) {
  auto kfn = ws_kernel_ptr<R, S, GRAD, CW, ASSIST>();
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (!bit || !(done.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, ws_smem_r<R>());
    if (e != cudaSuccess) return e;
    // clusters of up to 16 CTAs (tall planes); the occupancy query then reports how many fit
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
      cudaGetLastError();
    done.fetch_or(bit, std::memory_order_acq_rel);
  }
  *fn_out = reinterpret_cast<const void*>(kfn);
  return cudaSuccess;
}

// assist: the D group's W-box share for k = 9 (always on for k <= 7)
template <typename S, bool GRAD, int CW>
static cudaError_t ws_fn_r(int R, bool assist, const void** fn) {
  switch (R) {
    case 1: return ws_prepare<1, S, GRAD, CW, true>(fn);
    case 2: return ws_prepare<2, S, GRAD, CW, true>(fn);
    case 3: return ws_prepare<3, S, GRAD, CW, true>(fn);
    case 4: return assist ? ws_prepare<4, S, GRAD, CW, true>(fn) : ws_prepare<4, S, GRAD, CW, false>(fn);
    default: return cudaErrorInvalidValue;
  }
}

template <typename S, bool GRAD>
static cudaError_t ws_fn_cw(int R, int cw, bool assist, const void** fn) {
  return cw == 8 ? ws_fn_r<S, GRAD, 8>(R, assist, fn) : ws_fn_r<S, GRAD, 4>(R, assist, fn);
}

static cudaError_t ws_kernel_fn(int R, int dtype, bool grad, int cw, bool assist, const void** fn) {
  return with_dtype(dtype, [&](auto tag) {
    using S = decltype(tag);
    return grad ? ws_fn_cw<S, true>(R, cw, assist, fn) : ws_fn_cw<S, false>(R, cw, assist, fn);
  });
}

static int ws_smem_for(int R) {
  switch (R) {
    case 1: return ws_smem_r<1>();
    case 2: return ws_smem_r<2>();
    case 3: return ws_smem_r<3>();
    default: return ws_smem_r<4>();
  }
}

static int ws_max_clusters(const void* fn, int cy, int R) {
  static std::mutex mu;
  struct Key { int dev; int cy; const void* fn; int val; };
  static Key cache[128];
  static int ncache = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < ncache; ++i)
    if (cache[i].dev == dev && cache[i].cy == cy && cache[i].fn == fn) return cache[i].val;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(cy);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(unsigned(cy), 1, 1);
  cfg.blockDim = dim3(ws::NT, 1, 1);
  cfg.dynamicSmemBytes = size_t(ws_smem_for(R));
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess || n < 1) {
    cudaGetLastError();
    n = 0;
  }
  if (ncache < 128) cache[ncache++] = {dev, cy, fn, n};
  return n;
}

struct WsPlan {
  bool ok;
  int R;
  int cy;
  int tiles_x, tiles_y;
  int64_t total;
  int64_t nclusters;
  int64_t ipc;
  const void* fn;
  // Companion launch on the SMs the main launch leaves idle (clusters of 8 at one CTA per SM do not
  // tile every GPC): clusters of kCompanionCy CTAs over the last `b2` volumes, or, when the volumes
  // are too few for that, the last `z2` output planes of every volume, run concurrently on a second
  // stream. Both 0: none.
  int64_t b2;
  int64_t z2;
  int tiles_y2;
  int64_t total2, nclusters2, ipc2;
  int64_t parts() const { return int64_t(cy) * nclusters + int64_t(kCompanionCy) * nclusters2; }
  static constexpr int kCompanionCy = 2;
};

static WsPlan make_ws_plan(int64_t B, int64_t H, int64_t W, int k, int dtype, bool grad, int64_t z_begin,
                           int64_t z_end, const void* p, const void* t, const void* g) {
  WsPlan wp{false, k / 2, 0, 0, 0, 0, 0, 0, nullptr, 0, 0, 0, 0, 0, 0};
  const int choice = g_kernel_choice.load();
  if (choice == 1) return wp;
  // pointers unknown (workspace query): plan as for aligned tensors
  const int cw = (p == nullptr && t == nullptr) ? ((W % 8 == 0) ? 8 : (W % 4 == 0) ? 4 : 0)
                                                 : ws_chunk(W, dtype, p, t, g);
  if (cw == 0) return wp;
  // k = 9 compiles the kernel twice: with the D group's W-box share (it pays in clusters of up to 8
  // CTAs; measured: the MRI batch +3.7%) and without it (taller clusters: one 256^3 volume +4.7%).
  // Every occupancy query below is made on the variant that the launch of that cluster size uses.
  const void* fn = nullptr;
  const void* fn_tall = nullptr;
  if (ws_kernel_fn(k / 2, dtype, grad, cw, true, &fn) != cudaSuccess ||
      ws_kernel_fn(k / 2, dtype, grad, cw, false, &fn_tall) != cudaSuccess) {
    cudaGetLastError();
    return wp;
  }
  const int R = k / 2;
  int cy = int((H + ws::TY - 1) / ws::TY);
  if (cy > kWsMaxCluster) cy = kWsMaxCluster;
  int ty = ws::tile_count(int(H), ws::TY * cy, R, 1);
  const int tx = ws::tile_count(int(W), ws::SPAN, R, cw);
  int maxc = ws_max_clusters(fn, cy, R);
  if (maxc < 1) return wp;
  // A plane of 129 - 256 rows needs 2 - 3 overlapping row tiles in clusters of 8 but one in a taller
  // (non-portable) cluster, of which fewer fit: take the taller one when its row tiles per resident
  // cluster are fewer (every cluster advances one tile-plane per step whatever its height).
  if (H > int64_t(ws::TY) * kWsMaxCluster && H <= int64_t(ws::TY) * kWsMaxTall) {
    const int cyt = int((H + ws::TY - 1) / ws::TY);
    const int maxt = ws_max_clusters(fn_tall, cyt, R);
    if (maxt >= 1 && 1.0 / maxt < double(ty) / maxc) {
      cy = cyt;
      ty = 1;
      maxc = maxt;
      fn = fn_tall;
    }
  }
  const int64_t dz = z_end - z_begin;
  const int64_t min_ipc = 32;
  // Companion: when the main launch fills every cluster slot but leaves SMs idle, give the last b2
  // volumes (too few volumes: the last z2 planes of each) to clusters of 2 CTAs on those SMs. Their
  // span is 32 rows, so a plane costs ty2 tiles instead of ty; the split balances the two launches'
  // cluster-steps (resident clusters / row tiles per plane each).
  int64_t b2 = 0, z2 = 0, nc2 = 0;
  int ty2 = 0;
  if (cy >= 4 && B * int64_t(tx) * ty * dz >= min_ipc * maxc && g_companion.load() && !t_single_launch) {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess) {
      nc2 = (sms - int64_t(cy) * maxc) / WsPlan::kCompanionCy;
      const int maxc2 = ws_max_clusters(fn, WsPlan::kCompanionCy, R);
      if (nc2 > maxc2) nc2 = maxc2;
      if (nc2 >= 2) {
        ty2 = ws::tile_count(int(H), ws::TY * WsPlan::kCompanionCy, R, 1);
        const double r1 = double(maxc) / ty, r2 = double(nc2) / ty2;
        b2 = int64_t(double(B) * r2 / (r1 + r2) + 0.5);
        if (b2 > B - 1) b2 = B - 1;
        if (b2 < 1) {
          // too few volumes for a share of whole ones: the last planes of every volume instead; each
          // launch's segments start with a 2r-plane warm-up, so neither share may be tiny
          b2 = 0;
          z2 = int64_t(double(dz) * r2 / (r1 + r2) + 0.5);
          if (z2 < 8 || dz - z2 < 8) z2 = 0;
        }
      }
    }
    cudaGetLastError();
  }
  const int64_t total = (B - b2) * int64_t(tx) * ty * (dz - z2);  // b2 and z2 are never both set
  int64_t nc = (total + min_ipc - 1) / min_ipc;
  if (nc > maxc) nc = maxc;
  if (nc < 1) nc = 1;
  const int64_t ipc = (total + nc - 1) / nc;
  nc = (total + ipc - 1) / ipc;
  if (b2 > 0 || z2 > 0) {
    wp.b2 = b2;
    wp.z2 = z2;
    wp.tiles_y2 = ty2;
    wp.total2 = (b2 > 0 ? b2 * dz : B * z2) * int64_t(tx) * ty2;
    wp.ipc2 = (wp.total2 + nc2 - 1) / nc2;
    wp.nclusters2 = (wp.total2 + wp.ipc2 - 1) / wp.ipc2;
  }
  wp.ok = true;
  wp.cy = cy;
  wp.tiles_x = tx;
  wp.tiles_y = ty;
  wp.total = total;
  wp.nclusters = nc;
  wp.ipc = ipc;
  wp.fn = fn;
  return wp;
}

static cudaError_t launch_ws_grid(const WsPlan& wp, int cy, int64_t nclusters, const ws::Args& wa,
                                  cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(cy);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(unsigned(cy), unsigned(nclusters), 1);
  cfg.blockDim = dim3(ws::NT, 1, 1);
  cfg.dynamicSmemBytes = size_t(ws_smem_for(wp.R));
  cfg.stream = st;
  void* args[] = {const_cast<ws::Args*>(&wa)};
  return cudaLaunchKernelExC(&cfg, wp.fn, args);
}

// Stream for the companion launch and fork / join events (no timing), per host thread and device,
// made on first use outside stream capture and kept for the life of the thread (a stream captured into
// one thread's graph is never touched by another thread's call). Returns false when they cannot be
// had, in which case the caller runs the main launch over every volume.
static bool companion_resources(int dev, bool create, cudaStream_t* comp, cudaEvent_t* fork,
                                cudaEvent_t* join) {
  struct Res {
    cudaStream_t st = nullptr;
    cudaEvent_t ev[2] = {nullptr, nullptr};
  };
  thread_local Res res[64];
  if (dev < 0 || dev >= 64) return false;
  Res& r = res[dev];
  if (!r.st) {
    if (!create) return false;
    if (cudaEventCreateWithFlags(&r.ev[0], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&r.ev[1], cudaEventDisableTiming) != cudaSuccess ||
        cudaStreamCreateWithFlags(&r.st, cudaStreamNonBlocking) != cudaSuccess) {
      cudaGetLastError();
      if (r.ev[0]) cudaEventDestroy(r.ev[0]);
      if (r.ev[1]) cudaEventDestroy(r.ev[1]);
      r = Res();
      return false;
    }
  }
  *comp = r.st;
  *fork = r.ev[0];
  *join = r.ev[1];
  return true;
}

// Main launch on `st`; with a companion, the companion launch runs on the library's second stream,
// forked from and joined back into `st` (both legal under stream capture), so work queued on `st`
// after this call sees both. *nparts: the loss partials written, at wa.partials.
static cudaError_t launch_ws(const WsPlan& wp, const ws::Args& wa, cudaStream_t st, int64_t B, int64_t D,
                             int64_t H, int64_t W, int dtype, int64_t* nparts) {
  cudaStream_t comp = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  bool use2 = wp.b2 > 0 || wp.z2 > 0;
  if (use2) {
    // under stream capture only resources made earlier are used (no creation while capturing)
    int dev = 0;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    use2 = cudaGetDevice(&dev) == cudaSuccess && cudaStreamIsCapturing(st, &cs) == cudaSuccess &&
           companion_resources(dev, cs == cudaStreamCaptureStatusNone, &comp, &fork, &join);
    cudaGetLastError();
  }
  if (!use2) {
    // every volume in the main launch, over the same number of clusters (so the same partials)
    ws::Args a1 = wa;
    a1.total_items = B * int64_t(wp.tiles_x) * wp.tiles_y * (int64_t(wa.z_end) - wa.z_begin);
    a1.items_per_cluster = (a1.total_items + wp.nclusters - 1) / wp.nclusters;
    const int64_t nc = (a1.total_items + a1.items_per_cluster - 1) / a1.items_per_cluster;
    *nparts = int64_t(wp.cy) * nc;
    a1.n_parts = *nparts;
    return launch_ws_grid(wp, wp.cy, nc, a1, st);
  }
  *nparts = wp.parts();
  const size_t esz = dtype_size(dtype);
  ws::Args a1 = wa, a2 = wa;
  if (wp.z2 > 0) {  // every volume: the main launch takes planes [z_begin, zs), the companion [zs, z_end)
    const int zs = wa.z_end - int(wp.z2);
    a1.z_end = zs;
    a2.z_begin = zs;
    if (wa.g) {
      a2.g = static_cast<char*>(wa.g) + size_t(int64_t(zs - wa.z_begin) * H * W) * esz;
      a2.n_g = wa.n_g - int64_t(zs - wa.z_begin) * H * W;
    }
  } else {  // the main launch takes volumes [0, B - b2), the companion the rest
    const int64_t b1 = B - wp.b2;
    a2.p = static_cast<const char*>(wa.p) + size_t(b1 * D * H * W) * esz;
    a2.t = static_cast<const char*>(wa.t) + size_t(b1 * D * H * W) * esz;
    a2.n_in = wp.b2 * D * H * W;
    if (wa.g) {
      a2.g = static_cast<char*>(wa.g) + size_t(b1 * (int64_t(wa.z_end) - wa.z_begin) * H * W) * esz;
      a2.n_g = wp.b2 * (int64_t(wa.z_end) - wa.z_begin) * H * W;
    }
  }
  a1.n_parts = int64_t(wp.cy) * wp.nclusters;
  a2.n_parts = int64_t(WsPlan::kCompanionCy) * wp.nclusters2;
  cudaError_t e = cudaEventRecord(fork, st);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(comp, fork, 0);
  if (e == cudaSuccess) e = launch_ws_grid(wp, wp.cy, wp.nclusters, a1, st);
  if (e == cudaSuccess) {
    a2.partials = wa.partials + int64_t(wp.cy) * wp.nclusters;
    a2.clear_abort = 0;  // the main launch clears the word; both may set it
    a2.tiles_y = wp.tiles_y2;
    a2.span_y = ws::TY * WsPlan::kCompanionCy;
    a2.total_items = wp.total2;
    a2.items_per_cluster = wp.ipc2;
    e = launch_ws_grid(wp, WsPlan::kCompanionCy, wp.nclusters2, a2, comp);
  }
  if (e == cudaSuccess) e = cudaEventRecord(join, comp);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(st, join, 0);
  return e;
}

// ------------------------------------------------------------------------------------------------
// fixed scratch for callers that cannot allocate device memory (lncc_fused_forward_noalloc)
// ------------------------------------------------------------------------------------------------
// Room for this many fp64 partial sums (512 KiB); every GPU that loads the library holds it until
// the process exits. Each call's kernels write every partial they later read, so nothing needs
// clearing between calls; calls that overlap on the GPU share the array and race.
constexpr int64_t kNoAllocMaxPartials = 65536;
static __device__ __align__(256) double g_noalloc_partials[kNoAllocMaxPartials];

// Device address of g_noalloc_partials on the current device, looked up once per device. In host
// code the symbol is only a host-side stand-in, never a device address.
static int noalloc_scratch(double** out) {
  static std::mutex mu;
  static double* addr[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LNCC_ERR_CUDA;
  std::lock_guard<std::mutex> lk(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_partials) != cudaSuccess || p == nullptr) return LNCC_ERR_CUDA;
    addr[dev] = static_cast<double*>(p);
  }
  *out = addr[dev];
  return LNCC_OK;
}

// ---- materialising compat kernels (lncc_compat.cuh) ---------------------------------------------
template <int MODE, typename S>
static cudaError_t launch_compat(int R, const compat::Args& a, int64_t nblocks, cudaStream_t st) {
  const dim3 grid{unsigned(nblocks)}, block{unsigned(compat::NT)};
  switch (R) {
    case 1: compat::compat_kernel<1, MODE, S><<<grid, block, 0, st>>>(a); break;
    case 2: compat::compat_kernel<2, MODE, S><<<grid, block, 0, st>>>(a); break;
    case 3: compat::compat_kernel<3, MODE, S><<<grid, block, 0, st>>>(a); break;
    case 4: compat::compat_kernel<4, MODE, S><<<grid, block, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// Window of the materialising paths: cubic (k = kd = kh = kw in {3,5,7,9}, the compiled radii) or any
// kd x kh x kw with each side odd in 1 .. 9 (one instantiation of radius 4, the radii at run time).
struct Win {
  int kd, kh, kw;
  bool cubic() const { return kd == kh && kh == kw && valid_k(kd); }
};
static bool valid_side(int k) { return k >= 1 && k <= 9 && (k & 1); }
constexpr int kAnisoMaxR = 4;

template <int MODE, typename S>
static cudaError_t launch_compat_w(const Win& w, const compat::Args& a, int64_t nblocks, cudaStream_t st) {
  if (w.cubic()) return launch_compat<MODE, S>(w.kd / 2, a, nblocks, st);
  compat::compat_kernel<kAnisoMaxR, MODE, S, true><<<dim3(unsigned(nblocks)), dim3(compat::NT), 0, st>>>(a);
  return cudaGetLastError();
}

static int compat_plan(int64_t B, int64_t D, int64_t H, int64_t W, int k, compat::Args* a, int64_t* nblocks);
// As compat_plan, for a window of any odd sides in 1 .. 9 (sets the radii and n = kd*kh*kw).
static int compat_plan_w(int64_t B, int64_t D, int64_t H, int64_t W, const Win& w, compat::Args* a,
                         int64_t* nblocks) {
  if (!valid_side(w.kd) || !valid_side(w.kh) || !valid_side(w.kw)) return LNCC_ERR_KERNEL_SIZE;
  const int st = compat_plan(B, D, H, W, w.cubic() ? w.kd : 3, a, nblocks);
  if (st != LNCC_OK) return st;
  a->rd = w.kd / 2;
  a->rh = w.kh / 2;
  a->rw = w.kw / 2;
  a->n = float(w.kd * w.kh * w.kw);
  return LNCC_OK;
}

// Geometry and size checks shared by the three compat entry points; fills the tiling fields of `a`.
static int compat_plan(int64_t B, int64_t D, int64_t H, int64_t W, int k, compat::Args* a, int64_t* nblocks) {
  if (!valid_k(k)) return LNCC_ERR_KERNEL_SIZE;
  if (B < 1 || D < 1 || H < 1 || W < 1) return LNCC_ERR_BAD_ARG;
  if (D > INT32_MAX / 2 || H > INT32_MAX / 2 || W > INT32_MAX / 2) return LNCC_ERR_TOO_LARGE;
  a->n_elems = B * D * H * W;
  a->D = int(D);
  a->H = int(H);
  a->W = int(W);
  a->tiles_x = int((W + compat::TW - 1) / compat::TW);
  a->tiles_y = int((H + compat::TH - 1) / compat::TH);
  a->chunks = int((D + compat::ZCHUNK - 1) / compat::ZCHUNK);
  const int64_t nb = B * a->chunks * int64_t(a->tiles_y) * a->tiles_x;
  if (nb > INT32_MAX) return LNCC_ERR_TOO_LARGE;
  a->n = float(k * k * k);
  *nblocks = nb;
  return LNCC_OK;
}

// ---- checked build: every entry point reports range violations of its launches ----------------------
#ifdef LNCC_CHECKED
static int check_begin() {
  const unsigned long long z = 0;
  return cudaMemcpyToSymbol(g_check_violations, &z, sizeof(z)) == cudaSuccess ? LNCC_OK : LNCC_ERR_CUDA;
}
static int check_end(int status, cudaStream_t st) {
  if (status != LNCC_OK) return status;
  unsigned long long n = 0;
  if (cudaStreamSynchronize(st) != cudaSuccess ||
      cudaMemcpyFromSymbol(&n, g_check_violations, sizeof(n)) != cudaSuccess)
    return LNCC_ERR_CUDA;
  return n ? LNCC_ERR_CHECK : LNCC_OK;
}
#define LNCC_CHECKED_ENTRY(body, stream)   \
  do {                                     \
    const int cb_ = check_begin();         \
    if (cb_ != LNCC_OK) return cb_;        \
    return check_end((body), (stream));    \
  } while (0)
#endif

}  // namespace lncc

using namespace lncc;

extern "C" {

const char* lncc_strerror(int status) {
  switch (status) {
    case LNCC_OK: return "ok";
    case LNCC_ERR_BAD_ARG: return "fused_lncc: bad argument (null pointer, size or plane range)";
    case LNCC_ERR_KERNEL_SIZE: return "fused_lncc: kernel_size not supported (odd 3..9)";
    case LNCC_ERR_DTYPE: return "fused_lncc: float32, bfloat16 or float16 only";
    case LNCC_ERR_LAUNCH: return "fused_lncc: kernel launch failed";
    case LNCC_ERR_SMEM: return "fused_lncc: shared memory need exceeds this GPU's opt-in cap";
    case LNCC_ERR_WORKSPACE: return "fused_lncc: workspace missing or too small";
    case LNCC_ERR_CUDA: return "fused_lncc: CUDA runtime error";
    case LNCC_ERR_TOO_LARGE: return "fused_lncc: size exceeds the fixed maximum of this entry point";
    case LNCC_ERR_ABORTED: return "fused_lncc: a bounded wait in the kernel timed out; the results of that call are invalid";
    case LNCC_ERR_CHECK: return "fused_lncc: checked build: a kernel index left its array (the access was skipped)";
    default: return "fused_lncc: unknown status";
  }
}

int lncc_version(void) { return LNCC_VERSION_NUM; }

size_t lncc_workspace_bytes(int64_t B, int64_t D, int64_t H, int64_t W, int kernel_size, int dtype,
                            int64_t z_begin, int64_t z_end) {
  if (B < 1 || D < 1 || H < 1 || W < 1 || !valid_k(kernel_size)) return 0;
  if (z_begin < 0 || z_end > D || z_end <= z_begin) return 0;
  if (!valid_dtype(dtype)) return 0;
  // enough for either kernel (the choice also depends on pointer alignment, known only at launch)
  const Plan pl = make_plan(B, H, W, kernel_size, z_begin, z_end);
  size_t need = size_t(pl.nblocks) * sizeof(double);
  for (int gflag = 0; gflag < 2; ++gflag) {
    const WsPlan wp = make_ws_plan(B, H, W, kernel_size, dtype, gflag != 0, z_begin, z_end, nullptr, nullptr, nullptr);
    if (wp.ok && size_t(wp.parts()) * sizeof(double) > need) need = size_t(wp.parts()) * sizeof(double);
  }
  return need + kWsHeader;
}

static int impl_lncc_fused_forward(const void* pred, const void* target, int dtype, int64_t B, int64_t D, int64_t H,
                       int64_t W, int kernel_size, float smooth_dr, int64_t z_begin, int64_t z_end,
                       void* grad, float grad_scale, const float* grad_scale_dev, double* cc_sum_out,
                       float* loss_out, double loss_count, void* workspace, size_t workspace_bytes,
                       cudaStream_t stream) {
  if (!valid_k(kernel_size)) return LNCC_ERR_KERNEL_SIZE;
  if (!valid_dtype(dtype)) return LNCC_ERR_DTYPE;
  if (!pred || !target) return LNCC_ERR_BAD_ARG;
  if (B < 1 || D < 1 || H < 1 || W < 1) return LNCC_ERR_BAD_ARG;
  if (z_begin < 0 || z_end > D || z_end <= z_begin) return LNCC_ERR_BAD_ARG;
  if (D > INT32_MAX / 2 || H * W > INT32_MAX) return LNCC_ERR_TOO_LARGE;
  const size_t esz = dtype_size(dtype);
  if ((uintptr_t(pred) % esz) || (uintptr_t(target) % esz) || (grad && uintptr_t(grad) % esz))
    return LNCC_ERR_BAD_ARG;
  const Plan pl = make_plan(B, H, W, kernel_size, z_begin, z_end);
  if (pl.nblocks > INT32_MAX) return LNCC_ERR_TOO_LARGE;
  const WsPlan wp = make_ws_plan(B, H, W, kernel_size, dtype, grad != nullptr, z_begin, z_end, pred, target, grad);
  int64_t nparts = wp.ok ? wp.parts() : pl.nblocks;
  const size_t need = size_t(nparts) * sizeof(double) + kWsHeader;
  if (!workspace || workspace_bytes < need || (uintptr_t(workspace) % 8)) return LNCC_ERR_WORKSPACE;
  if (loss_out && !(loss_count > 0.0)) return LNCC_ERR_BAD_ARG;

  int dev = 0, cap = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return LNCC_ERR_CUDA;
  if (cudaDeviceGetAttribute(&cap, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return LNCC_ERR_CUDA;
  if (smem_needed(pl.R) > size_t(cap)) return LNCC_ERR_SMEM;

  SweepArgs a;
  a.p = pred;
  a.t = target;
  a.g = grad;
  a.partials = reinterpret_cast<double*>(static_cast<char*>(workspace) + kWsHeader);
  a.abort_word = static_cast<unsigned*>(workspace);
  a.n_in = B * D * H * W;
  a.n_g = grad ? B * (z_end - z_begin) * H * W : 0;
  a.n_parts = nparts;
  a.gscale_dev = grad_scale_dev;
  a.gscale = grad_scale;
  a.n = float(kernel_size * kernel_size * kernel_size);
  a.dr = smooth_dr;
  a.D = int(D);
  a.H = int(H);
  a.W = int(W);
  a.z_begin = int(z_begin);
  a.z_end = int(z_end);
  a.dchunk = pl.dchunk;
  a.tiles_w = pl.tiles_w;
  a.tiles_h = pl.tiles_h;
  a.nchunks = pl.nchunks;

  cudaError_t e;
  const bool g = grad != nullptr;
  if (wp.ok) {
    ws::Args wa;
    wa.p = pred;
    wa.t = target;
    wa.g = grad;
    wa.partials = a.partials;
    wa.abort_word = a.abort_word;
    wa.clear_abort = 1;
    wa.n_in = B * D * H * W;
    wa.n_g = grad ? B * (z_end - z_begin) * H * W : 0;
    wa.n_parts = nparts;
    wa.gscale_dev = grad_scale_dev;
    wa.gscale = grad_scale;
    wa.n = a.n;
    wa.dr = smooth_dr;
    wa.D = int(D);
    wa.H = int(H);
    wa.W = int(W);
    wa.z_begin = int(z_begin);
    wa.z_end = int(z_end);
    wa.tiles_x = wp.tiles_x;
    wa.tiles_y = wp.tiles_y;
    wa.span_y = ws::TY * wp.cy;
    wa.g_planes = int(z_end - z_begin);
    wa.total_items = wp.total;
    wa.items_per_cluster = wp.ipc;
    e = launch_ws(wp, wa, stream, B, D, H, W, dtype, &nparts);
  } else {
    e = with_dtype(dtype, [&](auto tag) {
      using S = decltype(tag);
      return g ? dispatch_r<S, true>(pl.R, a, pl.nblocks, stream) : dispatch_r<S, false>(pl.R, a, pl.nblocks, stream);
    });
  }
  if (e != cudaSuccess) return LNCC_ERR_LAUNCH;
  if (cc_sum_out || loss_out) {
    lncc_reduce_kernel<<<1, 1024, 0, stream>>>(a.partials, int(nparts), cc_sum_out, loss_out,
                                               loss_count > 0.0 ? loss_count : 1.0);
    if (cudaGetLastError() != cudaSuccess) return LNCC_ERR_LAUNCH;
  }
  return LNCC_OK;
}

int lncc_fused_forward_noalloc(const void* pred, const void* target, int dtype, int64_t B, int64_t D,
                               int64_t H, int64_t W, int kernel_size, float smooth_dr, int64_t z_begin,
                               int64_t z_end, void* grad, float grad_scale, const float* grad_scale_dev,
                               double* cc_sum_out, float* loss_out, double loss_count, cudaStream_t stream) {
  struct SingleLaunch {  // no companion launch: it would make a stream and events on first use
    SingleLaunch() { t_single_launch = true; }
    ~SingleLaunch() { t_single_launch = false; }
  } single;
  const size_t cap = size_t(kNoAllocMaxPartials) * sizeof(double);
  const size_t need = lncc_workspace_bytes(B, D, H, W, kernel_size, dtype, z_begin, z_end);
  if (need > cap) return LNCC_ERR_TOO_LARGE;
  double* scratch = nullptr;
  const int st = noalloc_scratch(&scratch);
  if (st != LNCC_OK) return st;
  // need == 0 means invalid arguments: the regular entry point reports the precise status. The
  // regular entry point re-plans with the real pointers; a plan needing more partials than the fixed
  // array holds is a size beyond this entry point's maximum, not a caller's workspace error.
  const int r = lncc_fused_forward(pred, target, dtype, B, D, H, W, kernel_size, smooth_dr, z_begin, z_end,
                                   grad, grad_scale, grad_scale_dev, cc_sum_out, loss_out, loss_count, scratch,
                                   cap, stream);
  return r == LNCC_ERR_WORKSPACE ? LNCC_ERR_TOO_LARGE : r;
}

int lncc_checked_build(void) {
#ifdef LNCC_CHECKED
  return 1;
#else
  return 0;
#endif
}

size_t lncc_peer_exchange_bytes(int world) {
  if (world < 1 || world > 32) return 0;
  return size_t(2) * size_t(world) * 2 * sizeof(uint64_t);
}

int lncc_peer_loss(const double* local_sum, void* const* slots, int rank, int world, uint64_t epoch, double count,
                   double* cc_sum_out, float* loss_out, unsigned* abort_word, cudaStream_t stream) {
  if (!local_sum || !slots || world < 1 || world > 32 || rank < 0 || rank >= world || epoch == 0 ||
      !(count > 0.0) || (uintptr_t(slots) % 8))
    return LNCC_ERR_BAD_ARG;
  lncc_peer_loss_kernel<<<1, 32, 0, stream>>>(local_sum, reinterpret_cast<uint64_t* const*>(slots), rank, world,
                                              epoch, count, cc_sum_out, loss_out, abort_word, ws::kWaitLimitNs);
  return cudaGetLastError() == cudaSuccess ? LNCC_OK : LNCC_ERR_LAUNCH;
}

int lncc_check_abort(const void* workspace, cudaStream_t stream) {
  if (!workspace || (uintptr_t(workspace) % 8)) return LNCC_ERR_BAD_ARG;
  unsigned w = 0;
  if (cudaMemcpyAsync(&w, workspace, sizeof(w), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return LNCC_ERR_CUDA;
  return w ? LNCC_ERR_ABORTED : LNCC_OK;
}

int lncc_wait_timeout_selftest(void* workspace, size_t workspace_bytes, unsigned limit_us, cudaStream_t stream) {
  if (!workspace || workspace_bytes < kWsHeader || (uintptr_t(workspace) % 8)) return LNCC_ERR_WORKSPACE;
  if (limit_us == 0 || limit_us > 10000000u) return LNCC_ERR_BAD_ARG;
  ws::wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(static_cast<unsigned*>(workspace),
                                                         (unsigned long long)limit_us * 1000ull);
  return cudaGetLastError() == cudaSuccess ? LNCC_OK : LNCC_ERR_LAUNCH;
}

int lncc_select_kernel(int which) {
  if (which < 0 || which > 3 || which == 2) return LNCC_ERR_BAD_ARG;
  g_kernel_choice.store(which);
  return LNCC_OK;
}

int lncc_set_companion(int enable) { return g_companion.exchange(enable ? 1 : 0); }

int lncc_launch_count(int64_t B, int64_t D, int64_t H, int64_t W, int kernel_size, int dtype, int64_t z_begin,
                      int64_t z_end, int grad) {
  // errors are negative so that they never read as a count
  if (!valid_k(kernel_size)) return -LNCC_ERR_KERNEL_SIZE;
  if (!valid_dtype(dtype)) return -LNCC_ERR_DTYPE;
  if (B < 1 || D < 1 || H < 1 || W < 1 || z_begin < 0 || z_end > D || z_end <= z_begin) return -LNCC_ERR_BAD_ARG;
  const WsPlan wp = make_ws_plan(B, H, W, kernel_size, dtype, grad != 0, z_begin, z_end, nullptr, nullptr, nullptr);
  return (wp.ok && (wp.b2 > 0 || wp.z2 > 0)) ? 2 : 1;
}

static int impl_lncc_maps_forward(const void* pred, const void* target, int dtype, int64_t B, int64_t D, int64_t H,
                      int64_t W, int kernel_size, float smooth_dr, float* ncc, float* A, float* Bc, float* Cc,
                      cudaStream_t stream) {
  if (!valid_dtype(dtype)) return LNCC_ERR_DTYPE;
  compat::Args a = {};
  int64_t nb = 0;
  const int st = compat_plan(B, D, H, W, kernel_size, &a, &nb);
  if (st != LNCC_OK) return st;
  if (!pred || !target) return LNCC_ERR_BAD_ARG;
  const size_t esz = dtype_size(dtype);
  if ((uintptr_t(pred) % esz) || (uintptr_t(target) % esz)) return LNCC_ERR_BAD_ARG;
  for (const float* m : {static_cast<const float*>(ncc), static_cast<const float*>(A),
                         static_cast<const float*>(Bc), static_cast<const float*>(Cc)})
    if (uintptr_t(m) % 4) return LNCC_ERR_BAD_ARG;
  a.in[0] = pred;
  a.in[1] = target;
  a.out[0] = ncc;
  a.out[1] = A;
  a.out[2] = Bc;
  a.out[3] = Cc;
  a.ndr = a.n * smooth_dr;
  const cudaError_t e = with_dtype(dtype, [&](auto tag) { return launch_compat<compat::MAPS, decltype(tag)>(kernel_size / 2, a, nb, stream); });
  return e == cudaSuccess ? LNCC_OK : LNCC_ERR_LAUNCH;
}

static int impl_lncc_maps_backward(const float* A, const float* Bc, const float* Cc, const void* pred, const void* target,
                       int dtype, int64_t B, int64_t D, int64_t H, int64_t W, int kernel_size, float scale,
                       void* grad, cudaStream_t stream) {
  if (!valid_dtype(dtype)) return LNCC_ERR_DTYPE;
  compat::Args a = {};
  int64_t nb = 0;
  const int st = compat_plan(B, D, H, W, kernel_size, &a, &nb);
  if (st != LNCC_OK) return st;
  if (!A || !Bc || !Cc || !pred || !target || !grad) return LNCC_ERR_BAD_ARG;
  const size_t esz = dtype_size(dtype);
  if ((uintptr_t(pred) % esz) || (uintptr_t(target) % esz) || (uintptr_t(grad) % esz)) return LNCC_ERR_BAD_ARG;
  if ((uintptr_t(A) % 4) || (uintptr_t(Bc) % 4) || (uintptr_t(Cc) % 4)) return LNCC_ERR_BAD_ARG;
  a.in[0] = A;
  a.in[1] = Bc;
  a.in[2] = Cc;
  a.p = pred;
  a.t = target;
  a.out[0] = grad;
  a.scale = scale;
  const cudaError_t e = with_dtype(dtype, [&](auto tag) { return launch_compat<compat::BWD, decltype(tag)>(kernel_size / 2, a, nb, stream); });
  return e == cudaSuccess ? LNCC_OK : LNCC_ERR_LAUNCH;
}

static int impl_lncc_box3d(const float* x, float* y, int64_t B, int64_t D, int64_t H, int64_t W, int kernel_size,
               cudaStream_t stream) {
  compat::Args a = {};
  int64_t nb = 0;
  const int st = compat_plan(B, D, H, W, kernel_size, &a, &nb);
  if (st != LNCC_OK) return st;
  if (!x || !y || (uintptr_t(x) % 4) || (uintptr_t(y) % 4)) return LNCC_ERR_BAD_ARG;
  a.in[0] = x;
  a.out[0] = y;
  const cudaError_t e = launch_compat<compat::BOX, float>(kernel_size / 2, a, nb, stream);
  return e == cudaSuccess ? LNCC_OK : LNCC_ERR_LAUNCH;
}

size_t lncc_loss_map_scratch_bytes(int64_t B, int64_t D, int64_t H, int64_t W) {
  if (B < 1 || D < 1 || H < 1 || W < 1) return 0;
  return size_t(3) * size_t(B) * size_t(D) * size_t(H) * size_t(W) * sizeof(float);
}

static int impl_lncc_loss_map_forward(const void* pred, const void* target, int dtype, int64_t B, int64_t D, int64_t H,
                          int64_t W, const Win& win, float smooth_dr, float* loss_map, cudaStream_t stream) {
  if (!valid_dtype(dtype)) return LNCC_ERR_DTYPE;
  compat::Args a = {};
  int64_t nb = 0;
  const int st = compat_plan_w(B, D, H, W, win, &a, &nb);
  if (st != LNCC_OK) return st;
  if (!pred || !target || !loss_map) return LNCC_ERR_BAD_ARG;
  const size_t esz = dtype_size(dtype);
  if ((uintptr_t(pred) % esz) || (uintptr_t(target) % esz) || (uintptr_t(loss_map) % 4)) return LNCC_ERR_BAD_ARG;
  a.in[0] = pred;
  a.in[1] = target;
  a.out[0] = loss_map;
  a.loss_map = 1;
  a.ndr = a.n * smooth_dr;
  const cudaError_t e = with_dtype(dtype, [&](auto tag) { return launch_compat_w<compat::MAPS, decltype(tag)>(win, a, nb, stream); });
  return e == cudaSuccess ? LNCC_OK : LNCC_ERR_LAUNCH;
}

static int impl_lncc_loss_map_backward(const float* grad_map, const void* pred, const void* target, int dtype, int64_t B,
                           int64_t D, int64_t H, int64_t W, const Win& win, float smooth_dr, void* grad,
                           float* scratch, size_t scratch_bytes, cudaStream_t stream) {
  if (!valid_dtype(dtype)) return LNCC_ERR_DTYPE;
  compat::Args a = {};
  int64_t nb = 0;
  const int st = compat_plan_w(B, D, H, W, win, &a, &nb);
  if (st != LNCC_OK) return st;
  if (!grad_map || !pred || !target || !grad) return LNCC_ERR_BAD_ARG;
  const size_t esz = dtype_size(dtype);
  if ((uintptr_t(pred) % esz) || (uintptr_t(target) % esz) || (uintptr_t(grad) % esz) ||
      (uintptr_t(grad_map) % 4))
    return LNCC_ERR_BAD_ARG;
  const size_t need = lncc_loss_map_scratch_bytes(B, D, H, W);
  if (!scratch || scratch_bytes < need || (uintptr_t(scratch) % 4)) return LNCC_ERR_WORKSPACE;
  const size_t nvox = need / (3 * sizeof(float));
  float* mA = scratch;
  float* mB = scratch + nvox;
  float* mC = scratch + 2 * nvox;
  // G-weighted adjoint maps at every voxel, then -(box(G*A) + 2p*box(G*Bc) + t*box(G*Cc))
  a.in[0] = pred;
  a.in[1] = target;
  a.out[1] = mA;
  a.out[2] = mB;
  a.out[3] = mC;
  a.wmap = grad_map;
  a.ndr = a.n * smooth_dr;
  cudaError_t e = with_dtype(dtype, [&](auto tag) { return launch_compat_w<compat::MAPS, decltype(tag)>(win, a, nb, stream); });
  if (e != cudaSuccess) return LNCC_ERR_LAUNCH;
  compat::Args b = a;
  b.in[0] = mA;
  b.in[1] = mB;
  b.in[2] = mC;
  b.p = pred;
  b.t = target;
  b.out[0] = grad;
  b.out[1] = b.out[2] = b.out[3] = nullptr;
  b.wmap = nullptr;
  b.scale = -1.f;
  e = with_dtype(dtype, [&](auto tag) { return launch_compat_w<compat::BWD, decltype(tag)>(win, b, nb, stream); });
  return e == cudaSuccess ? LNCC_OK : LNCC_ERR_LAUNCH;
}

// Non-cubic window: adjoint maps (A, Bc, Cc, fp32, in the scratch) and the per-block cc sums in one
// pass, the loss from those sums, then the maps backward for the gradient.
static size_t aniso_parts(int64_t B, int64_t D, int64_t H, int64_t W) {
  compat::Args a = {};
  int64_t nb = 0;
  return compat_plan(B, D, H, W, 3, &a, &nb) == LNCC_OK ? size_t(nb) : 0;
}

size_t lncc_aniso_scratch_bytes(int64_t B, int64_t D, int64_t H, int64_t W, int with_grad) {
  const size_t nb = aniso_parts(B, D, H, W);
  if (nb == 0) return 0;
  const size_t maps = with_grad ? size_t(3) * size_t(B) * size_t(D) * size_t(H) * size_t(W) * sizeof(float) : 0;
  return nb * sizeof(double) + maps;
}

static int impl_lncc_aniso_forward(const void* pred, const void* target, int dtype, int64_t B, int64_t D, int64_t H,
                                   int64_t W, const Win& win, float smooth_dr, void* grad, float grad_scale,
                                   const float* grad_scale_dev, double* cc_sum_out, float* loss_out,
                                   double loss_count, void* scratch, size_t scratch_bytes, cudaStream_t stream) {
  if (!valid_dtype(dtype)) return LNCC_ERR_DTYPE;
  compat::Args a = {};
  int64_t nb = 0;
  const int st = compat_plan_w(B, D, H, W, win, &a, &nb);
  if (st != LNCC_OK) return st;
  if (!pred || !target) return LNCC_ERR_BAD_ARG;
  const size_t esz = dtype_size(dtype);
  if ((uintptr_t(pred) % esz) || (uintptr_t(target) % esz) || (grad && uintptr_t(grad) % esz)) return LNCC_ERR_BAD_ARG;
  const size_t need = lncc_aniso_scratch_bytes(B, D, H, W, grad != nullptr);
  if (!scratch || scratch_bytes < need || (uintptr_t(scratch) % 8)) return LNCC_ERR_WORKSPACE;
  double* parts = static_cast<double*>(scratch);
  const size_t nvox = size_t(B) * size_t(D) * size_t(H) * size_t(W);
  float* maps = reinterpret_cast<float*>(parts + nb);
  a.in[0] = pred;
  a.in[1] = target;
  if (grad) {
    a.out[1] = maps;
    a.out[2] = maps + nvox;
    a.out[3] = maps + 2 * nvox;
  }
  a.partials = parts;
  a.n_parts = nb;
  a.ndr = a.n * smooth_dr;
  cudaError_t e = with_dtype(dtype, [&](auto tag) { return launch_compat_w<compat::MAPS, decltype(tag)>(win, a, nb, stream); });
  if (e != cudaSuccess) return LNCC_ERR_LAUNCH;
  if (cc_sum_out || loss_out) {
    lncc_reduce_kernel<<<1, 1024, 0, stream>>>(parts, int(nb), cc_sum_out, loss_out,
                                               loss_count > 0.0 ? loss_count : double(nvox));
    if (cudaGetLastError() != cudaSuccess) return LNCC_ERR_LAUNCH;
  }
  if (!grad) return LNCC_OK;
  compat::Args b = a;
  b.in[0] = a.out[1];
  b.in[1] = a.out[2];
  b.in[2] = a.out[3];
  b.p = pred;
  b.t = target;
  b.out[0] = grad;
  b.out[1] = b.out[2] = b.out[3] = nullptr;
  b.partials = nullptr;
  b.scale = grad_scale;
  b.scale_dev = grad_scale_dev;
  e = with_dtype(dtype, [&](auto tag) { return launch_compat_w<compat::BWD, decltype(tag)>(win, b, nb, stream); });
  return e == cudaSuccess ? LNCC_OK : LNCC_ERR_LAUNCH;
}

static int impl_lncc_scale_grad(void* grad, int dtype, int64_t n, const float* grad_out_dev, cudaStream_t stream) {
  if (!valid_dtype(dtype)) return LNCC_ERR_DTYPE;
  if (!grad || !grad_out_dev || n < 0) return LNCC_ERR_BAD_ARG;
  if (n == 0) return LNCC_OK;
  const int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  const int64_t cap = 8LL * sm_count_current();
  if (blocks > cap) blocks = cap;
  with_dtype(dtype, [&](auto tag) {
    using S = decltype(tag);
    lncc_scale_grad_kernel<S><<<unsigned(blocks), threads, 0, stream>>>(static_cast<S*>(grad), n, grad_out_dev);
    return 0;
  });
  return cudaGetLastError() == cudaSuccess ? LNCC_OK : LNCC_ERR_LAUNCH;
}

// ---- entry points (a checked build adds its range-violation report around each) ------------------
int lncc_fused_forward(const void* pred, const void* target, int dtype, int64_t B, int64_t D, int64_t H,
                       int64_t W, int kernel_size, float smooth_dr, int64_t z_begin, int64_t z_end,
                       void* grad, float grad_scale, const float* grad_scale_dev, double* cc_sum_out,
                       float* loss_out, double loss_count, void* workspace, size_t workspace_bytes,
                       cudaStream_t stream) {
#ifdef LNCC_CHECKED
  LNCC_CHECKED_ENTRY(impl_lncc_fused_forward(
      pred, target, dtype, B, D, H, W, kernel_size, smooth_dr, z_begin, z_end, grad, grad_scale,
      grad_scale_dev, cc_sum_out, loss_out, loss_count, workspace, workspace_bytes, stream), stream);
#else
  return impl_lncc_fused_forward(
      pred, target, dtype, B, D, H, W, kernel_size, smooth_dr, z_begin, z_end, grad, grad_scale,
      grad_scale_dev, cc_sum_out, loss_out, loss_count, workspace, workspace_bytes, stream);
#endif
}

int lncc_maps_forward(const void* pred, const void* target, int dtype, int64_t B, int64_t D, int64_t H,
                      int64_t W, int kernel_size, float smooth_dr, float* ncc, float* A, float* Bc, float* Cc,
                      cudaStream_t stream) {
#ifdef LNCC_CHECKED
  LNCC_CHECKED_ENTRY(impl_lncc_maps_forward(
      pred, target, dtype, B, D, H, W, kernel_size, smooth_dr, ncc, A, Bc, Cc, stream), stream);
#else
  return impl_lncc_maps_forward(pred, target, dtype, B, D, H, W, kernel_size, smooth_dr, ncc, A, Bc, Cc, stream);
#endif
}

int lncc_maps_backward(const float* A, const float* Bc, const float* Cc, const void* pred, const void* target,
                       int dtype, int64_t B, int64_t D, int64_t H, int64_t W, int kernel_size, float scale,
                       void* grad, cudaStream_t stream) {
#ifdef LNCC_CHECKED
  LNCC_CHECKED_ENTRY(impl_lncc_maps_backward(
      A, Bc, Cc, pred, target, dtype, B, D, H, W, kernel_size, scale, grad, stream), stream);
#else
  return impl_lncc_maps_backward(A, Bc, Cc, pred, target, dtype, B, D, H, W, kernel_size, scale, grad, stream);
#endif
}

int lncc_box3d(const float* x, float* y, int64_t B, int64_t D, int64_t H, int64_t W, int kernel_size,
               cudaStream_t stream) {
#ifdef LNCC_CHECKED
  LNCC_CHECKED_ENTRY(impl_lncc_box3d(x, y, B, D, H, W, kernel_size, stream), stream);
#else
  return impl_lncc_box3d(x, y, B, D, H, W, kernel_size, stream);
#endif
}

#ifdef LNCC_CHECKED
#define LNCC_ENTRY(body, stream) LNCC_CHECKED_ENTRY(body, stream)
#else
#define LNCC_ENTRY(body, stream) return (body)
#endif

int lncc_loss_map_forward(const void* pred, const void* target, int dtype, int64_t B, int64_t D, int64_t H,
                          int64_t W, int kernel_size, float smooth_dr, float* loss_map, cudaStream_t stream) {
  if (!valid_k(kernel_size)) return LNCC_ERR_KERNEL_SIZE;
  const Win win{kernel_size, kernel_size, kernel_size};
  LNCC_ENTRY(impl_lncc_loss_map_forward(pred, target, dtype, B, D, H, W, win, smooth_dr, loss_map, stream), stream);
}

int lncc_loss_map_backward(const float* grad_map, const void* pred, const void* target, int dtype, int64_t B,
                           int64_t D, int64_t H, int64_t W, int kernel_size, float smooth_dr, void* grad,
                           float* scratch, size_t scratch_bytes, cudaStream_t stream) {
  if (!valid_k(kernel_size)) return LNCC_ERR_KERNEL_SIZE;
  const Win win{kernel_size, kernel_size, kernel_size};
  LNCC_ENTRY(impl_lncc_loss_map_backward(grad_map, pred, target, dtype, B, D, H, W, win, smooth_dr, grad, scratch,
                                         scratch_bytes, stream),
             stream);
}

int lncc_aniso_forward(const void* pred, const void* target, int dtype, int64_t B, int64_t D, int64_t H, int64_t W,
                       int kd, int kh, int kw, float smooth_dr, void* grad, float grad_scale,
                       const float* grad_scale_dev, double* cc_sum_out, float* loss_out, double loss_count,
                       void* scratch, size_t scratch_bytes, cudaStream_t stream) {
  const Win win{kd, kh, kw};
  LNCC_ENTRY(impl_lncc_aniso_forward(pred, target, dtype, B, D, H, W, win, smooth_dr, grad, grad_scale, grad_scale_dev,
                                     cc_sum_out, loss_out, loss_count, scratch, scratch_bytes, stream),
             stream);
}

int lncc_aniso_loss_map_forward(const void* pred, const void* target, int dtype, int64_t B, int64_t D, int64_t H,
                                int64_t W, int kd, int kh, int kw, float smooth_dr, float* loss_map,
                                cudaStream_t stream) {
  const Win win{kd, kh, kw};
  LNCC_ENTRY(impl_lncc_loss_map_forward(pred, target, dtype, B, D, H, W, win, smooth_dr, loss_map, stream), stream);
}

int lncc_aniso_loss_map_backward(const float* grad_map, const void* pred, const void* target, int dtype, int64_t B,
                                 int64_t D, int64_t H, int64_t W, int kd, int kh, int kw, float smooth_dr, void* grad,
                                 float* scratch, size_t scratch_bytes, cudaStream_t stream) {
  const Win win{kd, kh, kw};
  LNCC_ENTRY(impl_lncc_loss_map_backward(grad_map, pred, target, dtype, B, D, H, W, win, smooth_dr, grad, scratch,
                                         scratch_bytes, stream),
             stream);
}

int lncc_scale_grad(void* grad, int dtype, int64_t n, const float* grad_out_dev, cudaStream_t stream) {
#ifdef LNCC_CHECKED
  LNCC_CHECKED_ENTRY(impl_lncc_scale_grad(grad, dtype, n, grad_out_dev, stream), stream);
#else
  return impl_lncc_scale_grad(grad, dtype, n, grad_out_dev, stream);
#endif
}

}  // extern "C"
