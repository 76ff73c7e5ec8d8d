// Materialising compat kernels: the reference extension's three entry points with the same outputs.
//
//   maps forward  (reference lncc_forward,  lncc3d.cu:127-161): pred, target -> four fp32 maps: ncc
//                 (clamped cc) and the adjoints A = dncc/dSp, Bc = dncc/dvar_p, Cc = dncc/dcross
//                 (lncc3d.cu:93-108);
//   maps backward (reference lncc_backward, lncc3d.cu:253-284): A, Bc, Cc, pred, target ->
//                 scale * (box(A) + 2*pred*box(Bc) + target*box(Cc)) in pred's dtype;
//   box3d         (reference box3d_sep_forward, lncc3d.cu:329-344): zero-padded k^3 box sum, fp32.
//
// These are for debugging and for code written against the reference's extension (its tests call
// lncc_forward / box3d_sep_forward directly). The training path is the fused kernel, which
// materialises nothing. The maps forward also serves the per-voxel loss (reduction 'none'): it can
// write 1 - ncc instead of ncc, and weight the adjoints by an upstream gradient map G at each voxel,
// so that the maps backward with scale -1 gives d(sum_v G(v) * (1 - ncc(v)))/dpred.
//
// One kernel template, three epilogues. A block owns a TH x TW tile of output columns (H, W) of one
// volume and a chunk of up to ZCHUNK output planes. Each thread owns a few columns of the
// (TH+2r) x (TW+2r) footprint and keeps their running D-window sums of the NF fields in registers:
// per output plane z it adds raw plane z+r and subtracts raw plane z-r-1 (re-read, L2 hits). The D
// sums are then boxed along H and along W in shared memory, and the epilogue sees the k^3 window sums
// at each output voxel. Raw planes outside the volume are zero padding, as in the reference.
#pragma once

namespace lncc {
namespace compat {

constexpr int TH = 16, TW = 32, NT = 256, ZCHUNK = 64;

enum Mode { MAPS = 0, BWD = 1, BOX = 2 };

template <int MODE> struct Fields;
template <> struct Fields<MAPS> { static constexpr int NRAW = 2, NF = 5; };  // p, t -> p, t, pp, tt, pt
template <> struct Fields<BWD> { static constexpr int NRAW = 3, NF = 3; };   // A, Bc, Cc
template <> struct Fields<BOX> { static constexpr int NRAW = 1, NF = 1; };   // x

struct Args {
  const void* in[3];   // MAPS: pred, target (S); BWD: A, Bc, Cc (fp32); BOX: x (fp32)
  const void* p;       // BWD: pred and target at the output voxel (S)
  const void* t;
  void* out[4];        // MAPS: ncc, A, Bc, Cc (fp32, each may be null); BWD: grad (S); BOX: y (fp32)
  const float* wmap;   // MAPS: null, or a (B, D, H, W) fp32 map multiplying A, Bc, Cc voxel by voxel
  int loss_map;        // MAPS: out[0] receives 1 - ncc instead of ncc
  int64_t n_elems;     // B * D * H * W (range checks of the checked build)
  int D, H, W;
  int tiles_x, tiles_y, chunks;
  float n, ndr, scale;
  const float* scale_dev;  // BWD: null, or a device float that also multiplies the gradient
  double* partials;    // MAPS: null, or one fp64 sum of the clamped cc per block (the loss)
  int64_t n_parts;     // entries writable at partials
  int rd, rh, rw;      // ANISO: window half-widths along D, H, W (0 .. R each)
};

template <typename S> __device__ __forceinline__ float ld(const S* p);
template <> __device__ __forceinline__ float ld<float>(const float* p) { return __ldg(p); }
template <> __device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(__ldg(p));
}
template <typename S> __device__ __forceinline__ void st(S* p, float v);
template <> __device__ __forceinline__ void st<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ float ld<__half>(const __half* p) { return __half2float(__ldg(p)); }
template <> __device__ __forceinline__ void st<__half>(__half* p, float v) { *p = __float2half_rn(v); }

// S: element type of pred/target (MAPS inputs, BWD output); the maps and box3d data are fp32.
// ANISO = false: the cubic window k = 2R + 1. ANISO = true: a kd x kh x kw window with the half-widths
// a.rd, a.rh, a.rw (each at most R, which sizes the shared arrays); n = kd * kh * kw comes in a.n.
template <int R, int MODE, typename S, bool ANISO = false>
__global__ void __launch_bounds__(NT) compat_kernel(const Args a) {
  constexpr int NF = Fields<MODE>::NF;
  constexpr int FHM = TH + 2 * R, FWM = TW + 2 * R, FPM = FHM * FWM;  // largest footprint
  constexpr int PPT = (FPM + NT - 1) / NT;
  __shared__ float DS[NF][FHM][FWM];  // D-window sums of the current output plane, footprint
  __shared__ float HS[NF][TH][FWM];   // after the H box
  __shared__ double red[NT / 32];
  // compile-time constants in the cubic instantiations
  const int rd = ANISO ? a.rd : R, rh = ANISO ? a.rh : R, rw = ANISO ? a.rw : R;
  const int kh = 2 * rh + 1, kw = 2 * rw + 1;
  const int FH = TH + 2 * rh, FW = TW + 2 * rw, FP = FH * FW;

  const int tid = threadIdx.x;
  int64_t bid = blockIdx.x;
  const int tx = int(bid % a.tiles_x); bid /= a.tiles_x;
  const int ty = int(bid % a.tiles_y); bid /= a.tiles_y;
  const int ch = int(bid % a.chunks); bid /= a.chunks;
  const int64_t b = bid;
  const int x0 = tx * TW, y0 = ty * TH;
  const int z0 = ch * ZCHUNK, z1 = min(z0 + ZCHUNK, a.D);
  const int64_t HW = int64_t(a.H) * a.W;
  const int64_t vol = b * int64_t(a.D) * HW;

  int64_t off[PPT];
  bool in[PPT];
#pragma unroll
  for (int j = 0; j < PPT; ++j) {
    const int i = tid + j * NT;
    const int gy = y0 - rh + i / FW, gx = x0 - rw + i % FW;
    in[j] = i < FP && gy >= 0 && gy < a.H && gx >= 0 && gx < a.W;
    off[j] = in[j] ? int64_t(gy) * a.W + gx : 0;
  }
  float s[PPT][NF];
#pragma unroll
  for (int j = 0; j < PPT; ++j)
#pragma unroll
    for (int f = 0; f < NF; ++f) s[j][f] = 0.f;

  // add (sgn = 1) or remove (sgn = -1) raw plane z; the same products either way, so they cancel
  auto accum = [&](int z, float sgn) {
    if (z < 0 || z >= a.D) return;
    const int64_t zo = vol + int64_t(z) * HW;
#pragma unroll
    for (int j = 0; j < PPT; ++j) {
      if (!in[j] || !LNCC_IN(zo + off[j], 1, a.n_elems)) continue;
      if (MODE == MAPS) {
        const float p = ld(static_cast<const S*>(a.in[0]) + zo + off[j]);
        const float t = ld(static_cast<const S*>(a.in[1]) + zo + off[j]);
        const float v[5] = {p, t, p * p, t * t, p * t};
#pragma unroll
        for (int f = 0; f < NF; ++f) s[j][f] += sgn * v[f];
      } else {
#pragma unroll
        for (int f = 0; f < NF; ++f) s[j][f] += sgn * ld(static_cast<const float*>(a.in[f]) + zo + off[j]);
      }
    }
  };

  double cc_acc = 0.0;  // MAPS with partials: this thread's sum of the clamped cc
  for (int z = z0 - rd; z < z0 + rd; ++z) accum(z, 1.f);
  for (int z = z0; z < z1; ++z) {
    accum(z + rd, 1.f);
    if (z > z0) accum(z - rd - 1, -1.f);
#pragma unroll
    for (int j = 0; j < PPT; ++j) {
      const int i = tid + j * NT;
      if (i < FP && LNCC_IN((i / FW) * FWM + i % FW, 1, FHM * FWM)) {
#pragma unroll
        for (int f = 0; f < NF; ++f) DS[f][i / FW][i % FW] = s[j][f];
      }
    }
    __syncthreads();
    for (int i = tid; i < TH * FW; i += NT) {  // H box
      const int r = i / FW, c = i % FW;
#pragma unroll
      for (int f = 0; f < NF; ++f) {
        float h = 0.f;
#pragma unroll
        for (int d = 0; d < kh; ++d) h += DS[f][r + d][c];
        if (LNCC_IN((r + kh - 1) * FWM + c, 1, FHM * FWM) && LNCC_IN(r * FWM + c, 1, TH * FWM)) HS[f][r][c] = h;
      }
    }
    __syncthreads();
    for (int i = tid; i < TH * TW; i += NT) {  // W box + epilogue
      const int r = i / TW, c = i % TW;
      const int y = y0 + r, x = x0 + c;
      if (y >= a.H || x >= a.W) continue;
      float w[NF];
#pragma unroll
      for (int f = 0; f < NF; ++f) {
        float h = 0.f;
#pragma unroll
        for (int d = 0; d < kw; ++d) h += HS[f][r][c + d];
        w[f] = h;
      }
      const int64_t o = vol + int64_t(z) * HW + int64_t(y) * a.W + x;
      if (!LNCC_IN(o, 1, a.n_elems) || !LNCC_IN(r * FWM + c + kw - 1, 1, TH * FWM)) continue;
      if (MODE == MAPS) {
        // n-scaled statistics (X = n*cross, VP = n*var_p, VT = n*var_t): the same cancellation of
        // constant inputs as the reference's division by n, and the same maps:
        //   ncc = X^2/(VP*VT), Cc = 2n*w, Bc = -n*w^2*VT, A = -2*w*(St - w*VT*Sp), w = X/(VP*VT)
        const float Sp = w[0], St = w[1], Spp = w[2], Stt = w[3], Spt = w[4];
        const float X = fmaf(a.n, Spt, -(Sp * St));
        const float VP = fmaxf(fmaf(a.n, Spp, -(Sp * Sp)), 0.f) + a.ndr;
        const float VT = fmaxf(fmaf(a.n, Stt, -(St * St)), 0.f) + a.ndr;
        const float den = VP * VT;
        float cc = (X * X) / den;
        float A = 0.f, Bc = 0.f, Cc = 0.f;
        if (cc < 1.f) {  // NaN falls through both branches: ncc NaN, adjoints zero (lncc3d.cu:101-107)
          const float wq = X / den;
          Cc = 2.f * a.n * wq;
          Bc = -a.n * (wq * wq) * VT;
          A = -2.f * wq * (St - wq * VT * Sp);
        } else if (cc >= 1.f) {
          cc = 1.f;
        }
        if (a.wmap) {
          const float gw = __ldg(a.wmap + o);
          A *= gw;
          Bc *= gw;
          Cc *= gw;
        }
        cc_acc += double(cc);
        if (a.out[0]) static_cast<float*>(a.out[0])[o] = a.loss_map ? 1.f - cc : cc;
        if (a.out[1]) static_cast<float*>(a.out[1])[o] = A;
        if (a.out[2]) static_cast<float*>(a.out[2])[o] = Bc;
        if (a.out[3]) static_cast<float*>(a.out[3])[o] = Cc;
      } else if (MODE == BWD) {
        const float p = ld(static_cast<const S*>(a.p) + o), t = ld(static_cast<const S*>(a.t) + o);
        const float sc = a.scale_dev ? a.scale * __ldg(a.scale_dev) : a.scale;
        st(static_cast<S*>(a.out[0]) + o, sc * (w[0] + 2.f * p * w[1] + t * w[2]));
      } else {
        static_cast<float*>(a.out[0])[o] = w[0];
      }
    }
    // the next plane's DS writes follow this thread's W pass; its H pass follows the next barrier
  }
  if (MODE == MAPS && a.partials) {  // block sum of the clamped cc, in a fixed order
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cc_acc += __shfl_down_sync(0xffffffffu, cc_acc, o);
    if ((tid & 31) == 0) red[tid >> 5] = cc_acc;
    __syncthreads();
    if (tid == 0) {
      double t = 0.0;
      for (int w = 0; w < NT / 32; ++w) t += red[w];
      if (LNCC_IN(blockIdx.x, 1, a.n_parts)) a.partials[blockIdx.x] = t;
    }
  }
}

}  // namespace compat
}  // namespace lncc
