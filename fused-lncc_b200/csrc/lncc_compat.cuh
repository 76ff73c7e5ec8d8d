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

// S: element type of pred/target (MAPS inputs, BWD output); the maps and box3d data are fp32.
template <int R, int MODE, typename S>
__global__ void __launch_bounds__(NT) compat_kernel(const Args a) {
  constexpr int NF = Fields<MODE>::NF;
  constexpr int K = 2 * R + 1;
  constexpr int FH = TH + 2 * R, FW = TW + 2 * R, FP = FH * FW;
  constexpr int PPT = (FP + NT - 1) / NT;
  __shared__ float DS[NF][FH][FW];  // D-window sums of the current output plane, footprint
  __shared__ float HS[NF][TH][FW];  // after the H box

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
    const int gy = y0 - R + i / FW, gx = x0 - R + i % FW;
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

  for (int z = z0 - R; z < z0 + R; ++z) accum(z, 1.f);
  for (int z = z0; z < z1; ++z) {
    accum(z + R, 1.f);
    if (z > z0) accum(z - R - 1, -1.f);
#pragma unroll
    for (int j = 0; j < PPT; ++j) {
      const int i = tid + j * NT;
      if (i < FP && LNCC_IN(i, 1, FH * FW)) {
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
        for (int d = 0; d < K; ++d) h += DS[f][r + d][c];
        if (LNCC_IN((r + K - 1) * FW + c, 1, FH * FW) && LNCC_IN(r * FW + c, 1, TH * FW)) HS[f][r][c] = h;
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
        for (int d = 0; d < K; ++d) h += HS[f][r][c + d];
        w[f] = h;
      }
      const int64_t o = vol + int64_t(z) * HW + int64_t(y) * a.W + x;
      if (!LNCC_IN(o, 1, a.n_elems) || !LNCC_IN(r * FW + c + K - 1, 1, TH * FW)) continue;
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
        if (a.out[0]) static_cast<float*>(a.out[0])[o] = a.loss_map ? 1.f - cc : cc;
        if (a.out[1]) static_cast<float*>(a.out[1])[o] = A;
        if (a.out[2]) static_cast<float*>(a.out[2])[o] = Bc;
        if (a.out[3]) static_cast<float*>(a.out[3])[o] = Cc;
      } else if (MODE == BWD) {
        const float p = ld(static_cast<const S*>(a.p) + o), t = ld(static_cast<const S*>(a.t) + o);
        st(static_cast<S*>(a.out[0]) + o, a.scale * (w[0] + 2.f * p * w[1] + t * w[2]));
      } else {
        static_cast<float*>(a.out[0])[o] = w[0];
      }
    }
    // the next plane's DS writes follow this thread's W pass; its H pass follows the next barrier
  }
}

}  // namespace compat
}  // namespace lncc
