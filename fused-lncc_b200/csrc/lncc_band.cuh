// Band kernel: the fast path of liblncc_sm100 for volumes with W <= 128, W % 4 == 0, H <= 256.
//
// A thread-block cluster of CY = ceil(H/16) CTAs covers one whole H x W plane of a volume; CTA
// `rank` owns rows [16*rank, 16*rank+16) and all W columns, and the cluster walks the volume along D.
// Halo rows in H are not recomputed: they are read from the neighbouring CTA's shared memory
// (DSMEM) after a cluster barrier. Halos in W do not exist (a CTA spans the full row) and halos in D
// are the running sums carried from plane to plane.
//
// Two thread layouts are used in turn:
//   row layout (RL)   : warp w <-> row w of the band, lane l <-> columns 4l..4l+3 (float4)
//   column layout (CL): thread <-> one column and a run of rows
// Per stat plane c (raw planes c-r..c+r):
//   A  [RL] D running sums of p, t, p*p, t*t, p*t (old raw plane re-read from L2), W box by warp
//           shuffles -> DW (5 fields) in shared memory
//   B  [CL] H box of DW -> the five window sums -> cc (loss partial) and the three adjoint fields
//           -> ADJ
//   C  [CL] H box of ADJ -> AH
// The R boundary rows of DW and ADJ are also written ("pushed") into the neighbour CTAs' halo rows
// through DSMEM when they are produced, so B and C read only local shared memory.
//   D  [RL] W box of AH by shuffles, D running sum through a k-deep ring of boxed adjoint planes
//           held in tensor memory (TMEM, private per thread) -> dL/dpred of output plane c-r
// Steps are software-pipelined with ONE split cluster barrier per step c:
//   A(c) -> arrive | prefetch, D(c-2) | wait -> B(c), C(c-1) -> __syncthreads
// DW and ADJ are double-buffered by step parity, so a buffer is rewritten only two steps after its
// remote readers have passed a barrier. AH is double-buffered too where shared memory allows (r <= 3):
// D(c-2) reads it between arrive and wait while C(c-1) writes it after the wait. With one AH buffer
// (r = 4) a CTA barrier after the wait keeps C(c-1) behind every D(c-2) of the CTA. Only the warps that pushed rows into a neighbour arrive with
// a cluster-scope release; the others fence at CTA scope and arrive relaxed. Global loads are issued
// after the arrive so that no fence waits for them.
#pragma once

#include <cooperative_groups.h>

namespace lncc {
namespace band {

namespace cg = cooperative_groups;

constexpr int TH = 16;          // rows per CTA (one warp per row in RL)
constexpr int NT = 32 * TH;     // 512 threads
constexpr int WMAX = 128;       // 32 lanes x 4 columns
constexpr int TMEM_COLS = 512;  // whole TMEM of the SM: one CTA per SM

struct BandArgs {
  const void* p;
  const void* t;
  void* g;
  double* partials;
  const float* gscale_dev;
  float gscale;
  float n;
  float dr;
  int D, H, W;
  int z_begin, z_end;
  int64_t total_planes;       // B * (z_end - z_begin)
  int64_t planes_per_cluster;
};

// DW and ADJ hold the CTA's own rows at [R, R+TH) plus R halo rows on each side: rows [0, R) are
// pushed by the CTA above (its last R rows), rows [R+TH, TH+2R) by the CTA below. Halo rows with no
// neighbour stay zero (the volume's zero padding).
// AH buffers: two where they fit in the 227 KB a CTA may use
template <int R>
constexpr int AH_BUFS = R <= 3 ? 2 : 1;
template <int R>
struct Smem {
  float DW[2][5][TH + 2 * R][WMAX];
  float ADJ[2][3][TH + 2 * R][WMAX];
  float AH[AH_BUFS<R>][3][TH][WMAX];
  double red[NT / 32];
  uint32_t tmem_base;
};
// Every variant takes more than half of an SM's shared memory, so each CTA is alone on its SM and
// may allocate all 512 TMEM columns without waiting for another CTA.
template <int R>
constexpr int smem_bytes() { return int((sizeof(Smem<R>) + 1023) / 1024 * 1024); }
static_assert(smem_bytes<1>() > 116 * 1024, "band smem: one CTA per SM");
static_assert(smem_bytes<1>() <= 227 * 1024 && smem_bytes<2>() <= 227 * 1024 && smem_bytes<3>() <= 227 * 1024 &&
                  smem_bytes<4>() <= 227 * 1024,
              "band smem: 227 KB per CTA");

template <typename S>
struct Vec4;
template <>
struct Vec4<float> {
  static __device__ __forceinline__ float4 load(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
  static __device__ __forceinline__ void store(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
};
template <>
struct Vec4<__nv_bfloat16> {
  static __device__ __forceinline__ float4 load(const __nv_bfloat16* p) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
    const float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
    return make_float4(fa.x, fa.y, fb.x, fb.y);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float4 v) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = u;
  }
};

__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive for a warp that wrote no other CTA's shared memory since its last arrive: a CTA-scope fence
// orders its local shared-memory writes, and the arrive itself is relaxed. A cluster-scope release
// (cluster_arrive) waits for every outstanding store and is the dominant cost of a plane step.
__device__ __forceinline__ void cluster_arrive_local() {
  asm volatile("fence.acq_rel.cta;" ::: "memory");
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

// ---- TMEM (tensor memory) used as a per-thread ring buffer ----------------------------------------
__device__ __forceinline__ void tmem_st12(uint32_t ta, const float (&v)[12]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(ta),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
      : "memory");
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(ta + 8),
               "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
               "r"(__float_as_uint(v[11]))
               : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Issue a 12-column load; the registers are valid only after tmem_ld_wait(u), which names them as
// operands so that no use can be scheduled before the wait.
__device__ __forceinline__ void tmem_ld12_issue(uint32_t ta, uint32_t (&u)[12]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]),
                 "=r"(u[7])
               : "r"(ta)
               : "memory");
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11])
               : "r"(ta + 8)
               : "memory");
}
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&u)[12]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(u[0]), "+r"(u[1]), "+r"(u[2]), "+r"(u[3]), "+r"(u[4]), "+r"(u[5]), "+r"(u[6]),
                 "+r"(u[7]), "+r"(u[8]), "+r"(u[9]), "+r"(u[10]), "+r"(u[11])
               :
               : "memory");
}

// W box of a float4 run per lane (columns 4l..4l+3) with half-width R, zero outside [0, 4*nlanes).
template <int R>
__device__ __forceinline__ float4 wbox(float4 v, int lane) {
  static_assert(R >= 1 && R <= 4, "R");
  const float x[4] = {v.x, v.y, v.z, v.w};
  float lft[4], rgt[4];  // only the R values next to this lane's run are fetched
#pragma unroll
  for (int i = 0; i < R; ++i) {
    lft[4 - R + i] = __shfl_up_sync(0xffffffffu, x[4 - R + i], 1);
    rgt[i] = __shfl_down_sync(0xffffffffu, x[i], 1);
  }
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < R; ++i) lft[4 - R + i] = 0.f;
  }
  if (lane == 31) {
#pragma unroll
    for (int i = 0; i < R; ++i) rgt[i] = 0.f;
  }
  // window elements e[-R .. 3+R]
  float e[4 + 2 * R];
#pragma unroll
  for (int i = 0; i < R; ++i) e[i] = lft[4 - R + i];
#pragma unroll
  for (int i = 0; i < 4; ++i) e[R + i] = x[i];
#pragma unroll
  for (int i = 0; i < R; ++i) e[R + 4 + i] = rgt[i];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 2 * R + 1; ++i) s += e[i];
  float o[4];
  o[0] = s;
#pragma unroll
  for (int q = 1; q < 4; ++q) {
    s += e[q + 2 * R] - e[q - 1];
    o[q] = s;
  }
  return make_float4(o[0], o[1], o[2], o[3]);
}

template <int R, typename S, bool GRAD, int NSEG>
__global__ void __launch_bounds__(NT, 1) lncc_band_kernel(const BandArgs a) {
  constexpr int K = 2 * R + 1;
  constexpr int L = TH / NSEG;          // CL rows per task
  constexpr int NCL = WMAX * NSEG;      // CL threads
  static_assert(NCL <= NT, "CL threads");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  using Smem = band::Smem<R>;
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int rank = blockIdx.x;            // cluster rank == band index along H
  const int nrank = gridDim.x;            // cluster size
  const int D = a.D, H = a.H, W = a.W;
  const int64_t HW = int64_t(H) * W;
  const float nf = a.n, ndr = a.n * a.dr;
  const int Dout = a.z_end - a.z_begin;

  // ---- TMEM: 512 columns; warp w uses lanes 32*(w%4).., columns 128*(w/4) .. +128 -----------------
  if (warp == 0) {
    const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(&sm.tmem_base));
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = sm.tmem_base + (uint32_t(32 * (warp & 3)) << 16) + uint32_t(128 * (warp >> 2));

  // neighbour shared memory (DSMEM); rank -1 / nrank have no neighbour (zero padding)
  Smem* up = rank > 0 ? cluster.map_shared_rank(&sm, rank - 1) : nullptr;
  Smem* dn = rank + 1 < nrank ? cluster.map_shared_rank(&sm, rank + 1) : nullptr;
  // zero the halo rows (those without a neighbour are never written); the first cluster barrier
  // below orders these stores before any neighbour's first push
  for (int i = tid; i < 2 * (5 + 3) * 2 * R * WMAX; i += NT) {
    const int col = i % WMAX, rr = (i / WMAX) % (2 * R), f = (i / (WMAX * 2 * R)) % 8, bb = i / (WMAX * 2 * R * 8);
    const int row = rr < R ? rr : TH + rr;
    if (f < 5) sm.DW[bb][f][row][col] = 0.f;
    else sm.ADJ[bb][f - 5][row][col] = 0.f;
  }
  cluster.sync();

  // RL ownership
  const int y_rl = rank * TH + warp;
  const int x_rl = 4 * lane;
  const bool rl_in = (y_rl < H) && (x_rl < W);
  const int64_t rl_off = rl_in ? int64_t(y_rl) * W + x_rl : 0;
  // CL ownership
  const int cl_col = tid % WMAX, cl_seg = tid / WMAX;
  const bool cl_thread = tid < NCL;
  const int cl_r0 = cl_seg * L;
  const bool cl_in_col = cl_thread && cl_col < W;
  // Warps that push rows into a neighbour CTA (DW in A, ADJ in B) arrive with cluster-scope release
  // semantics; the others only need CTA scope. The condition is uniform across each warp.
  const bool pushes_remote = (warp < R) || (warp >= TH - R) ||
                             (cl_thread && (cl_r0 < R || cl_r0 + L > TH - R));

  float gs = 0.f;
  if (GRAD) gs = 2.f * a.gscale * (a.gscale_dev ? __ldg(a.gscale_dev) : 1.f);
  float acc = 0.f;

  int64_t g0 = int64_t(blockIdx.y) * a.planes_per_cluster;
  const int64_t g1 = min(g0 + a.planes_per_cluster, a.total_planes);
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
  while (g0 < g1) {
    const int64_t b = g0 / Dout;
    const int zs = a.z_begin + int(g0 - b * Dout);
    const int64_t rem = g1 - b * Dout;
    const int ze = a.z_begin + int(rem < Dout ? rem : int64_t(Dout));
    g0 = b * Dout + (ze - a.z_begin);
    const S* __restrict__ P = reinterpret_cast<const S*>(a.p) + b * D * HW;
    const S* __restrict__ T = reinterpret_cast<const S*>(a.t) + b * D * HW;
    S* __restrict__ G = GRAD ? reinterpret_cast<S*>(a.g) + b * int64_t(Dout) * HW : nullptr;

    // ---- D running sums (RL registers), warm-up over raw planes [zs-2R, zs) ------------------------
    float4 s5[5];
#pragma unroll
    for (int f = 0; f < 5; ++f) s5[f] = zero4;
    float4 t3[3];
#pragma unroll
    for (int f = 0; f < 3; ++f) t3[f] = zero4;
    auto raw_ok = [&](int z) { return rl_in && z >= 0 && z < D; };
    auto add_plane = [&](float4 p, float4 t, float sgn) {
      s5[0].x = fmaf(sgn, p.x, s5[0].x); s5[0].y = fmaf(sgn, p.y, s5[0].y);
      s5[0].z = fmaf(sgn, p.z, s5[0].z); s5[0].w = fmaf(sgn, p.w, s5[0].w);
      s5[1].x = fmaf(sgn, t.x, s5[1].x); s5[1].y = fmaf(sgn, t.y, s5[1].y);
      s5[1].z = fmaf(sgn, t.z, s5[1].z); s5[1].w = fmaf(sgn, t.w, s5[1].w);
      s5[2].x = fmaf(sgn * p.x, p.x, s5[2].x); s5[2].y = fmaf(sgn * p.y, p.y, s5[2].y);
      s5[2].z = fmaf(sgn * p.z, p.z, s5[2].z); s5[2].w = fmaf(sgn * p.w, p.w, s5[2].w);
      s5[3].x = fmaf(sgn * t.x, t.x, s5[3].x); s5[3].y = fmaf(sgn * t.y, t.y, s5[3].y);
      s5[3].z = fmaf(sgn * t.z, t.z, s5[3].z); s5[3].w = fmaf(sgn * t.w, t.w, s5[3].w);
      s5[4].x = fmaf(sgn * p.x, t.x, s5[4].x); s5[4].y = fmaf(sgn * p.y, t.y, s5[4].y);
      s5[4].z = fmaf(sgn * p.z, t.z, s5[4].z); s5[4].w = fmaf(sgn * p.w, t.w, s5[4].w);
    };
    for (int z = zs - 2 * R; z < zs; ++z) {
      if (raw_ok(z)) add_plane(Vec4<S>::load(P + z * HW + rl_off), Vec4<S>::load(T + z * HW + rl_off), 1.f);
    }

    const int c0 = zs - R, c_end = ze + R;  // stat planes [c0, c_end)
    float4 pn = zero4, tn = zero4, po = zero4, to = zero4;  // raw planes for the next A
    if (raw_ok(c0 + R)) {
      pn = Vec4<S>::load(P + (c0 + R) * HW + rl_off);
      tn = Vec4<S>::load(T + (c0 + R) * HW + rl_off);
    }
    float4 pc = zero4, tc = zero4;  // pred/target of the output plane of the next D

    // D [RL]: W box of AH, D running sum through the TMEM ring, gradient of output plane c-R
    auto phase_D = [&](int c, float4 pcv, float4 tcv) {
      const int it = c - c0;
      const int ahb = AH_BUFS<R> == 2 ? (it & 1) : 0;  // C(c) wrote AH[(c - c0) & 1]
      const uint32_t ta = tmem + uint32_t(12 * (it % K));
      uint32_t u[12];
      const bool has_old = it >= K;
      tmem_wait_st();  // the previous plane's store has landed before any read
      if (has_old) tmem_ld12_issue(ta, u);
      float v[12];
#pragma unroll
      for (int f = 0; f < 3; ++f) {
        const float4 w4 = wbox<R>(*reinterpret_cast<const float4*>(&sm.AH[ahb][f][warp][x_rl]), lane);
        v[4 * f + 0] = w4.x; v[4 * f + 1] = w4.y; v[4 * f + 2] = w4.z; v[4 * f + 3] = w4.w;
      }
      if (has_old) {
        tmem_ld_wait(u);
      } else {
#pragma unroll
        for (int i = 0; i < 12; ++i) u[i] = 0u;
      }
      tmem_st12(ta, v);
      float* tt = reinterpret_cast<float*>(t3);
#pragma unroll
      for (int i = 0; i < 12; ++i) tt[i] += v[i] - __uint_as_float(u[i]);
      const int o = c - R;
      if (o >= zs && o < ze && rl_in) {
        // d(sum cc)/dp = 2*(n*t*box(c) - n*p*box(b) - box(a)); fields a=0, b=1, c=2
        float4 gq;
        gq.x = gs * fmaf(nf, fmaf(tcv.x, t3[2].x, -pcv.x * t3[1].x), -t3[0].x);
        gq.y = gs * fmaf(nf, fmaf(tcv.y, t3[2].y, -pcv.y * t3[1].y), -t3[0].y);
        gq.z = gs * fmaf(nf, fmaf(tcv.z, t3[2].z, -pcv.z * t3[1].z), -t3[0].z);
        gq.w = gs * fmaf(nf, fmaf(tcv.w, t3[2].w, -pcv.w * t3[1].w), -t3[0].w);
        Vec4<S>::store(G + int64_t(o - a.z_begin) * HW + rl_off, gq);
      }
    };

    // B [CL]: H box of DW[buf] (halo rows from neighbours) -> stats -> cc, adjoints -> ADJ[buf]
    auto phase_B = [&](int c, int buf) {
      const bool c_in = (c >= 0) && (c < D);
      const bool c_own = c_in && c >= zs && c < ze;
      float s[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
      float win[5][2 * R + 1];
      const float* dwp = &sm.DW[buf][0][cl_r0][cl_col];  // extended row cl_r0 = own row cl_r0 - R
      constexpr int FS = (TH + 2 * R) * WMAX;            // field stride
#pragma unroll
      for (int q = 0; q < L + 2 * R; ++q) {
        float v[5];
#pragma unroll
        for (int f = 0; f < 5; ++f) v[f] = dwp[f * FS + q * WMAX];
#pragma unroll
        for (int f = 0; f < 5; ++f) {
          s[f] += v[f];
          if (q >= 2 * R + 1) s[f] -= win[f][q % (2 * R + 1)];
          win[f][q % (2 * R + 1)] = v[f];
        }
        if (q >= 2 * R) {
          const int r = cl_r0 + q - 2 * R;
          const int y = rank * TH + r;
          const bool in = c_in && cl_in_col && y < H;
          const float Sp = s[0], St = s[1], Spp = s[2], Stt = s[3], Spt = s[4];
          const float X = fmaf(nf, Spt, -(Sp * St));
          const float VP = fmaxf(fmaf(nf, Spp, -(Sp * Sp)), 0.f) + ndr;
          const float VT = fmaxf(fmaf(nf, Stt, -(St * St)), 0.f) + ndr;
          float rden;
          asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(rden) : "f"(VP * VT));
          const float wq = X * rden;
          const float cc = X * wq;
          if (in && c_own) acc += (cc >= 1.f) ? 1.f : cc;
          if (GRAD) {
            const bool live = in && (cc < 1.f);  // NaN and cc >= 1: zero adjoints (lncc3d.cu:100-107)
            const float wv = wq * VT;
            const float av[3] = {live ? wq * fmaf(-wv, Sp, St) : 0.f, live ? wq * wv : 0.f, live ? wq : 0.f};
#pragma unroll
            for (int f = 0; f < 3; ++f) sm.ADJ[buf][f][R + r][cl_col] = av[f];
            // push boundary rows into the neighbours' halo rows
            if (r < R && up != nullptr) {
#pragma unroll
              for (int f = 0; f < 3; ++f) up->ADJ[buf][f][R + TH + r][cl_col] = av[f];
            }
            if (r >= TH - R && dn != nullptr) {
#pragma unroll
              for (int f = 0; f < 3; ++f) dn->ADJ[buf][f][r - (TH - R)][cl_col] = av[f];
            }
          }
        }
      }
    };

    // C [CL]: H box of ADJ[buf] (halo rows from neighbours) -> AH
    auto phase_C = [&](int c, int buf) {
      (void)c;
      const int ahb = AH_BUFS<R> == 2 ? buf : 0;  // buf = (c - c0) & 1
      float s[3] = {0.f, 0.f, 0.f};
      float win[3][2 * R + 1];
      const float* adp = &sm.ADJ[buf][0][cl_r0][cl_col];
      constexpr int FS = (TH + 2 * R) * WMAX;
#pragma unroll
      for (int q = 0; q < L + 2 * R; ++q) {
        float v[3];
#pragma unroll
        for (int f = 0; f < 3; ++f) v[f] = adp[f * FS + q * WMAX];
#pragma unroll
        for (int f = 0; f < 3; ++f) {
          s[f] += v[f];
          if (q >= 2 * R + 1) s[f] -= win[f][q % (2 * R + 1)];
          win[f][q % (2 * R + 1)] = v[f];
        }
        if (q >= 2 * R) {
          const int r = cl_r0 + q - 2 * R;
#pragma unroll
          for (int f = 0; f < 3; ++f) sm.AH[ahb][f][r][cl_col] = s[f];
        }
      }
    };

    // Software pipeline, one cluster barrier per step:
    //   step c:  A(c) -> arrive | prefetch, D(c-2) | wait -> B(c), C(c-1) -> __syncthreads
    // DW and ADJ are double-buffered by step parity, AH (local) too when AH_BUFS<R> == 2.
    for (int c = c0; c <= c_end + 1; ++c) {
      const int buf = (c - c0) & 1;
      if (c < c_end) {
        add_plane(pn, tn, 1.f);
        add_plane(po, to, -1.f);
#pragma unroll
        for (int f = 0; f < 5; ++f) {
          const float4 w4 = wbox<R>(s5[f], lane);
          *reinterpret_cast<float4*>(&sm.DW[buf][f][R + warp][x_rl]) = w4;
          // push boundary rows into the neighbours' halo rows (remote shared memory)
          if (warp < R && up != nullptr) *reinterpret_cast<float4*>(&up->DW[buf][f][R + TH + warp][x_rl]) = w4;
          if (warp >= TH - R && dn != nullptr)
            *reinterpret_cast<float4*>(&dn->DW[buf][f][warp - (TH - R)][x_rl]) = w4;
        }
      }
      // release covers the DW pushes (and the ADJ pushes of the previous B); global loads are issued
      // after it so that the fence never waits on them
      if (pushes_remote) cluster_arrive();
      else cluster_arrive_local();
      pn = tn = po = to = zero4;
      if (c + 1 < c_end) {
        if (raw_ok(c + 1 + R)) {
          pn = Vec4<S>::load(P + (c + 1 + R) * HW + rl_off);
          tn = Vec4<S>::load(T + (c + 1 + R) * HW + rl_off);
        }
        if (raw_ok(c - R)) {
          po = Vec4<S>::load(P + (c - R) * HW + rl_off);
          to = Vec4<S>::load(T + (c - R) * HW + rl_off);
        }
      }
      float4 pcn = zero4, tcn = zero4;
      if (GRAD) {
        const int o = c - 1 - R;  // output plane of D(c-1), run in the next step
        if (c - 1 >= c0 && o >= zs && o < ze && rl_in) {
          pcn = Vec4<S>::load(P + o * HW + rl_off);
          tcn = Vec4<S>::load(T + o * HW + rl_off);
        }
        if (c - 2 >= c0) phase_D(c - 2, pc, tc);
      }
      pc = pcn;
      tc = tcn;
      cluster_wait();
      if (AH_BUFS<R> == 1) __syncthreads();  // every D(c-2) of the CTA has read AH
      if (cl_thread) {
        if (c < c_end) phase_B(c, buf);
        if (GRAD && c - 1 >= c0 && c - 1 < c_end) phase_C(c - 1, buf ^ 1);
      }
      __syncthreads();
    }
  }
  tmem_wait_st();

  // ---- teardown: nobody may leave while a neighbour can still read its shared memory ---------------
  double dacc = acc;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dacc += __shfl_down_sync(0xffffffffu, dacc, o);
  if (lane == 0) sm.red[warp] = dacc;
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster.sync();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(sm.tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
  if (tid == 0) {
    double s = 0.0;
    for (int w = 0; w < NT / 32; ++w) s += sm.red[w];
    a.partials[int64_t(blockIdx.y) * gridDim.x + blockIdx.x] = s;
  }
}

}  // namespace band
}  // namespace lncc
