// Warp-specialised cluster kernel: the fast path of liblncc_sm100 (fused LNCC loss + dL/dpred).
//
// A thread-block cluster of CY CTAs covers a span of 16*CY rows x 128 columns of the H x W plane; CTA
// `rank` owns span rows [16*rank, 16*rank + 16). The cluster walks D one plane per step. Planes wider
// or taller than one span are cut into tiles whose spans overlap by 2*(k/2) columns / rows (the halo
// of the two-level stencil), and the walk covers (volume, tile, plane) items.
//
// Each CTA runs four warp groups (128 threads each) that hand planes to one another through shared
// memory, paced by mbarriers instead of CTA-wide barriers:
//   A   (warps 0-3)  thread <-> one row, 16 columns. Keeps D running sums of p, t, p*p, t*t, 2*p*t in
//                    tensor memory (TMEM), updated with the raw plane entering and the one leaving the
//                    window (both loaded one step ahead), boxes them along W with warp shuffles and
//                    stores them (DW) for the step's stat plane (for k <= 7 fields 0-2 only; the D
//                    warp with the same TMEM lanes and rows boxes fields 3-4). The CTA's first and last
//                    2r rows are then sent to the neighbouring CTAs' halo rows by bulk copies (TMA
//                    engine, one per warp and neighbour, completion counted in bytes on the receiver's
//                    barrier), so no CTA recomputes another CTA's rows.
//   BC  (warps 4-11) two threads per column, each for half of the CTA's rows: H box of DW over
//                    8 + 4r rows -> the five window sums -> cc (loss partial) and the three adjoint
//                    fields on 8 + 2r rows -> H box of the adjoints -> AH for its 8 rows.
//   D   (warps 12-15) thread <-> one row, 16 columns. W box of AH by shuffles, D running sum through a
//                    k-deep ring of boxed adjoint planes in TMEM, then the gradient of output plane
//                    c - r.
// DW and AH are double-buffered by step parity. mbarriers per buffer: dw_full (this CTA's A warps have
// written and the neighbours' halo bytes have landed), dw_empty (BC of this CTA and of both
// neighbours have read), ah_full, ah_empty; per pair of A warp w and D warp 12 + w: ya (the step's
// running sums are in TMEM) and xd (the D warp's fields are written). Every wait is bounded: after
// kWaitLimitNs the CTA sets an abort flag, every role of the CTA leaves its loops without arriving
// on a barrier again, and the CTA's loss partial becomes NaN.
//
// Statistics are kept multiplied by n = k^3 (see lncc_sm100.cu): X = n*Spt - Sp*St,
// VP = max(n*Spp - Sp^2, 0) + n*dr, VT likewise, w = X / (VP*VT), cc = X*w, and with wv = w*VT the
// adjoints a = w*(St - wv*Sp), b = w*wv, c = w give d(sum cc)/dp = 2*(n*t*box(c) - n*p*box(b) - box(a)).
// The running sum of p*t is kept doubled: the D update adds (p_in+p_out)(t_in-t_out) +
// (p_in-p_out)(t_in+t_out) = 2*(p_in*t_in - p_out*t_out).
#pragma once

#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "lncc_check.cuh"

namespace lncc {
namespace ws {

namespace cg = cooperative_groups;

constexpr int TY = 16;                // rows per CTA
constexpr int LPR = 8;                // lanes per row in the row-layout groups (A, D)
constexpr int VW = 16;                // columns per lane
constexpr int SPAN = LPR * VW;        // 128 columns per span
constexpr int NT = 512;               // 4 warp groups
constexpr int TMEM_COLS = 512;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

struct Args {
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
  int tiles_x, tiles_y;
  int span_y;                 // 16 * cluster size
  int g_planes;               // planes per volume of the gradient array (a launch may fill part of it)
  int64_t total_items;        // B * tiles_y * tiles_x * (z_end - z_begin)
  int64_t items_per_cluster;
  unsigned* abort_word;       // workspace word: set to 1 by a CTA whose bounded wait ran out
  int clear_abort;            // this launch's first CTA zeroes abort_word at its start
  int64_t n_in;               // elements readable from p and t (range checks of the checked build)
  int64_t n_g;                // elements writable at g
  int64_t n_parts;            // partials writable at partials
};

template <int R>
struct Geo {
  static constexpr int K = 2 * R + 1;
  static constexpr int ER = TY + 4 * R;  // DW rows: 2R halo rows above, 16 own, 2R below
  // TMEM columns per lane (the A and D threads of a warp quadrant share its 32 lanes):
  static constexpr uint32_t TM_RING = 0;    // D group: ring of K boxed adjoint planes, 48 columns each
  static constexpr uint32_t TM_A = 432;     // A group: D running sums, 5 fields x 16 columns
  // D group: running sums (3 fields x 16 columns) in TMEM where they fit (k <= 7), else in registers
  static constexpr bool DSUM_TMEM = TM_RING + 48 * K + 48 <= TM_A;
  static constexpr uint32_t TM_DSUM = TM_RING + 48 * K;
  static_assert(TM_RING + 48 * K <= TM_A && TM_A + 80 <= TMEM_COLS, "TMEM budget");
};

template <int R>
struct Smem {
  float dw[2][Geo<R>::ER][5][SPAN];  // W-boxed D sums (Sp, St, Spp, Stt, 2*Spt) per row, chunk-swizzled
  float ah[2][3][TY][SPAN];          // H-boxed adjoints (a, b, c) of the CTA's own rows
  unsigned long long bar[16];        // dw_full[2], dw_empty[2], ah_full[2], ah_empty[2], xd[4], ya[4]
  double red[8];                     // BC warps' loss partials
  uint32_t tmem_base;
  int abort_flag;
};
template <int R>
constexpr int smem_bytes() { return int((sizeof(Smem<R>) + 1023) / 1024 * 1024); }
// More than half of an SM's shared memory: one CTA per SM, so the 512-column TMEM allocation never
// waits for another CTA.
static_assert(smem_bytes<1>() > 116 * 1024, "ws smem: one CTA per SM");
static_assert(smem_bytes<4>() <= 227 * 1024, "ws smem: 227 KB per CTA");

enum { BAR_DW_FULL = 0, BAR_DW_EMPTY = 2, BAR_AH_FULL = 4, BAR_AH_EMPTY = 6, BAR_XD = 8, BAR_YA = 12 };

// Physical float offset of logical column x in a 128-float row. The 16-byte chunks of each 128-byte
// group are permuted (chunk ^= group & 3) so that the eight lanes of a row in the row layout, whose
// 16-byte accesses are 64 bytes apart, hit eight different bank groups; a warp of the column layout
// reading 32 consecutive columns still touches one 128-byte group.
__device__ __forceinline__ int swz(int x) {
  const int c = x >> 2;
  const int pc = (c & ~7) | ((c & 7) ^ ((c >> 3) & 3));
  return (pc << 2) | (x & 3);
}
// Physical float offset of logical chunk c (4 columns).
__device__ __forceinline__ int swz_chunk(int c) { return ((c & ~7) | ((c & 7) ^ ((c >> 3) & 3))) << 2; }

// ---- element access --------------------------------------------------------------------------------
// Two packed 16-bit elements (bf16 or fp16, in one 32-bit word) <-> float2.
template <typename S>
struct Pair16;
template <>
struct Pair16<__nv_bfloat16> {
  static __device__ __forceinline__ float2 to2(uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
  }
  static __device__ __forceinline__ uint32_t from2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <>
struct Pair16<__half> {
  static __device__ __forceinline__ float2 to2(uint32_t w) { return __half22float2(*reinterpret_cast<const __half2*>(&w)); }
  static __device__ __forceinline__ uint32_t from2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

template <typename S>
struct IO {  // 16-bit types: four elements in 8 bytes
  static __device__ __forceinline__ float4 ld(const S* p) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    const float2 a = Pair16<S>::to2(u.x), b = Pair16<S>::to2(u.y);
    return make_float4(a.x, a.y, b.x, b.y);
  }
  static __device__ __forceinline__ void st(S* p, float4 v) {
    *reinterpret_cast<uint2*>(p) = make_uint2(Pair16<S>::from2(v.x, v.y), Pair16<S>::from2(v.z, v.w));
  }
};

template <>
struct IO<float> {
  static __device__ __forceinline__ float4 ld(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
  static __device__ __forceinline__ void st(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
};

// Chunk of CW = 4 or 8 consecutive elements <-> CW/4 float4. CW = 8 uses one 256-bit access for fp32
// (ld/st .v8.f32, 32-byte aligned) and one 128-bit access for bf16 / fp16: with 16 columns per lane, a lane's
// two 8-column chunks fill whole 32-byte sectors, where 4-column chunks fill only half of each.
template <typename S, int CW>
struct Chunk;
template <>
struct Chunk<float, 4> {
  static __device__ __forceinline__ void ld(const float* p, float4* o) { o[0] = IO<float>::ld(p); }
  static __device__ __forceinline__ void st(float* p, const float4* v) { IO<float>::st(p, v[0]); }
};
template <typename S>
struct Chunk<S, 4> {  // 16-bit types
  static __device__ __forceinline__ void ld(const S* p, float4* o) { o[0] = IO<S>::ld(p); }
  static __device__ __forceinline__ void st(S* p, const float4* v) { IO<S>::st(p, v[0]); }
};
template <>
struct Chunk<float, 8> {
  static __device__ __forceinline__ void ld(const float* p, float4* o) {
    asm("ld.global.nc.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=f"(o[0].x), "=f"(o[0].y), "=f"(o[0].z), "=f"(o[0].w), "=f"(o[1].x), "=f"(o[1].y), "=f"(o[1].z),
                   "=f"(o[1].w)
                 : "l"(p));
  }
  static __device__ __forceinline__ void st(float* p, const float4* v) {
    asm volatile("st.global.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "f"(v[0].x), "f"(v[0].y), "f"(v[0].z),
                 "f"(v[0].w), "f"(v[1].x), "f"(v[1].y), "f"(v[1].z), "f"(v[1].w)
                 : "memory");
  }
};
template <typename S>
struct Chunk<S, 8> {  // 16-bit types: one 128-bit access
  static __device__ __forceinline__ void ld(const S* p, float4* o) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const float2 a = Pair16<S>::to2(u.x), b = Pair16<S>::to2(u.y), c = Pair16<S>::to2(u.z), d = Pair16<S>::to2(u.w);
    o[0] = make_float4(a.x, a.y, b.x, b.y);
    o[1] = make_float4(c.x, c.y, d.x, d.y);
  }
  static __device__ __forceinline__ void st(S* p, const float4* v) {
    *reinterpret_cast<uint4*>(p) = make_uint4(Pair16<S>::from2(v[0].x, v[0].y), Pair16<S>::from2(v[0].z, v[0].w),
                                              Pair16<S>::from2(v[1].x, v[1].y), Pair16<S>::from2(v[1].z, v[1].w));
  }
};

// ---- packed f32x2 arithmetic (sm_100) ------------------------------------------------------------------
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 sub2(float2 a, float2 b) { return __fadd2_rn(a, make_float2(-b.x, -b.y)); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// ---- mbarriers -----------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count) : "memory");
}
// Arrive on this CTA's barrier with CTA-scope release (orders this thread's prior shared-memory
// writes for waiters of the same CTA); a cluster-scope release costs ~300 cycles more.
__device__ __forceinline__ void mbar_arrive_cta(uint32_t a) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(a)
      : "memory");
}
// As mbar_arrive_cta, and the current phase also waits for `bytes` more of asynchronous (bulk copy)
// arrivals.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t a, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
// Relaxed arrive on the barrier at the same offset in CTA `rank`: used to report that this thread has
// finished READING a buffer that the other CTA will overwrite. Every read result has been consumed by
// instructions issued before the arrive, so the reads are complete when it is issued.
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t a, uint32_t rank) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(ra) : "memory");
}
// Bulk copy (TMA engine) of `bytes` from this CTA's shared memory to another CTA's; completion is
// signalled on the destination CTA's barrier `mbar_cluster` (complete_tx). Addresses 16-B aligned.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                                  uint32_t mbar_cluster) {
  if (!LNCC_IN_SMEM(src_cta, bytes)) return;
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst_cluster),
      "r"(src_cta), "r"(bytes), "r"(mbar_cluster)
      : "memory");
}
// Acquire at CTA scope, as for any transaction barrier: the barrier is in this CTA's shared memory, and
// the bytes the neighbours' bulk copies write here are visible once their complete_tx has been counted.
__device__ __forceinline__ bool mbar_test(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Slow path of mbar_wait: poll for at most kWaitLimitNs; on timeout set the CTA's abort flag, after
// which every wait of the CTA returns at once and the roles leave their loops (NaN loss partial).
__device__ __forceinline__ void mbar_wait_slow(uint32_t a, uint32_t parity, volatile int* abort_flag,
                                               unsigned long long limit_ns = kWaitLimitNs) {
  const unsigned long long t0 = global_ns();
  for (;;) {
    if (mbar_test(a, parity)) return;
    if (*abort_flag) return;
    if (global_ns() - t0 > limit_ns) {
      *abort_flag = 1;
      return;
    }
  }
}
// Wait for the phase of `parity` of the barrier at `a` to complete (bounded, see mbar_wait_slow).
__device__ __forceinline__ void mbar_wait(uint32_t a, uint32_t parity, volatile int* abort_flag) {
  if (!mbar_test(a, parity)) mbar_wait_slow(a, parity, abort_flag);
}

// ---- TMEM, used as per-thread storage (lane = thread of the warp quadrant) ------------------------------
// TMEM column ranges are warp-uniform, so a checked build skips a bad access for the whole warp.
#define LNCC_TM_OK(ta, n) LNCC_IN((ta) & 0xffffu, n, TMEM_COLS)
__device__ __forceinline__ void tm_ld16(uint32_t ta, float (&v)[16]) {
  if (!LNCC_TM_OK(ta, 16)) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = 0.f;
    return;
  }
  uint32_t u[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
        "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15])
      : "r"(ta)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(u[0]), "+r"(u[1]), "+r"(u[2]), "+r"(u[3]), "+r"(u[4]), "+r"(u[5]), "+r"(u[6]),
                 "+r"(u[7]), "+r"(u[8]), "+r"(u[9]), "+r"(u[10]), "+r"(u[11]), "+r"(u[12]), "+r"(u[13]),
                 "+r"(u[14]), "+r"(u[15])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(u[i]);
}
__device__ __forceinline__ void tm_st16(uint32_t ta, const float (&v)[16]) {
  if (!LNCC_TM_OK(ta, 16)) return;
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(ta),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tm_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 16-column load without the wait; the registers are valid only after tm_wait_ld16 names them.
__device__ __forceinline__ void tm_ld16_issue(uint32_t ta, uint32_t (&u)[16]) {
  if (!LNCC_TM_OK(ta, 16)) {
#pragma unroll
    for (int i = 0; i < 16; ++i) u[i] = 0u;
    return;
  }
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
        "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15])
      : "r"(ta));
}
// Waits for every outstanding TMEM load of the thread; naming the registers keeps their uses after it.
__device__ __forceinline__ void tm_wait_ld16(uint32_t (&u)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(u[0]), "+r"(u[1]), "+r"(u[2]), "+r"(u[3]), "+r"(u[4]), "+r"(u[5]), "+r"(u[6]),
                 "+r"(u[7]), "+r"(u[8]), "+r"(u[9]), "+r"(u[10]), "+r"(u[11]), "+r"(u[12]), "+r"(u[13]),
                 "+r"(u[14]), "+r"(u[15]));
}
__device__ __forceinline__ void tm_st8(uint32_t ta, const uint32_t (&u)[8]) {
  if (!LNCC_TM_OK(ta, 8)) return;
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(ta), "r"(u[0]),
               "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7])
               : "memory");
}
__device__ __forceinline__ void tm_st4(uint32_t ta, float4 v) {
  if (!LNCC_TM_OK(ta, 4)) return;
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(ta), "r"(__float_as_uint(v.x)),
               "r"(__float_as_uint(v.y)), "r"(__float_as_uint(v.z)), "r"(__float_as_uint(v.w))
               : "memory");
}

__device__ __forceinline__ void sts4(uint32_t addr, float4 v) {
  if (!LNCC_IN_SMEM(addr, 16)) return;
  asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ uint32_t mapa_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Empty asm naming a float4 as read-write: arithmetic on it cannot be scheduled before this point, so
// loads issued early (prefetch) are not waited for earlier than intended.
__device__ __forceinline__ void reg_fence(float4& v) {
  asm volatile("" : "+f"(v.x), "+f"(v.y), "+f"(v.z), "+f"(v.w));
}

// W box (half-width R) of the 16 columns of lane q of an 8-lane row; columns beyond the row's span are
// zero. Halo values come from the neighbouring lanes by shuffles. emit(j, float4) receives output
// columns 4j..4j+3 as soon as they are complete, so that at most four outputs are held at a time.
template <int R, typename Emit>
__device__ __forceinline__ void wbox16(const float (&v)[16], int q, Emit&& emit) {
  float lh[R], rh[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    lh[i] = __shfl_up_sync(0xffffffffu, v[16 - R + i], 1, LPR);
    rh[i] = __shfl_down_sync(0xffffffffu, v[i], 1, LPR);
  }
  if (q == 0) {
#pragma unroll
    for (int i = 0; i < R; ++i) lh[i] = 0.f;
  }
  if (q == LPR - 1) {
#pragma unroll
    for (int i = 0; i < R; ++i) rh[i] = 0.f;
  }
  auto E = [&](int j) -> float { return j < 0 ? lh[j + R] : (j < 16 ? v[j] : rh[j - 16]); };
  float s = E(-R);
#pragma unroll
  for (int j = -R + 1; j <= R; ++j) s += E(j);
  float o[4];
  o[0] = s;
#pragma unroll
  for (int i = 1; i < 16; ++i) {
    s += E(i + R) - E(i - R - 1);
    o[i & 3] = s;
    if ((i & 3) == 3) emit(i >> 2, make_float4(o[0], o[1], o[2], o[3]));
  }
}

// Output range [o0, o1) and span origin of tile t along an axis of `extent` voxels, for spans of
// `span` voxels and stencil half-width R. One tile when the axis fits in a span. Otherwise the first
// tile starts at the volume edge (no halo needed there) and the others start `halo` before their
// first output; `align` rounds the output boundaries (4 along W so that 16-byte chunks never straddle
// a tile boundary).
__host__ __device__ __forceinline__ void tile_geom(int t, int extent, int span, int R, int align, int& base,
                                                   int& o0, int& o1) {
  if (extent <= span) {
    base = 0;
    o0 = 0;
    o1 = extent;
    return;
  }
  const int halo = (2 * R + align - 1) / align * align;
  const int first = (span - 2 * R) / align * align;
  const int step = (span - halo - 2 * R) / align * align;
  if (t == 0) {
    base = 0;
    o0 = 0;
    o1 = first;
    return;
  }
  o0 = first + (t - 1) * step;
  o1 = o0 + step < extent ? o0 + step : extent;
  base = o0 - halo;
}
__host__ __device__ __forceinline__ int tile_count(int extent, int span, int R, int align) {
  if (extent <= span) return 1;
  const int halo = (2 * R + align - 1) / align * align;
  const int first = (span - 2 * R) / align * align;
  const int step = (span - halo - 2 * R) / align * align;
  return 1 + (extent - first + step - 1) / step;
}

// Geometry of one work segment: output planes [zs, ze) of volume b, tile (ty, tx).
struct Seg {
  int64_t b;
  int zs, ze;
  int yb, oy0, oy1;  // span row origin, output rows
  int xb, ox0, ox1;  // span column origin, output columns
};

// ASSIST: the D group boxes two of the five DW fields for the A group (always with the D running sums
// in TMEM, k <= 7; a choice of the launch for k = 9, where they live in registers).
template <int R, typename S, bool GRAD, int CW, bool ASSIST = true>
__global__ void __launch_bounds__(NT, 1) lncc_ws_kernel(const Args a) {
  constexpr int NCH = VW / CW;  // global-memory chunks per lane
  constexpr int K = Geo<R>::K;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  using SM = Smem<R>;
  SM& sm = *reinterpret_cast<SM*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int role = warp >> 2;  // 0 A, 1 BC0, 2 BC1, 3 D
  const int rank = int(blockIdx.x), nrank = int(gridDim.x);
  const bool has_up = rank > 0, has_dn = rank + 1 < nrank;
  const int D = a.D, H = a.H, W = a.W;
  const int64_t HW = int64_t(H) * W;
  const int Dout = a.z_end - a.z_begin;
  // every wait below is bounded by seconds, so this clear precedes any CTA's abort record
  if (a.clear_abort && a.abort_word && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) *a.abort_word = 0u;
  volatile int* abort_flag = &sm.abort_flag;
  const uint32_t bar0 = smem_addr(&sm.bar[0]);
  auto bar = [&](int which, int i) -> uint32_t { return bar0 + uint32_t(8 * (which + i)); };

  // ---- set-up ----------------------------------------------------------------------------------------
  if (tid == 0) {
    const uint32_t nb = 8u * (1u + (has_up ? 1u : 0u) + (has_dn ? 1u : 0u));
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(BAR_DW_FULL, i), 4);   // local A warps (+ the halo rows' bulk-copy bytes)
      mbar_init(bar(BAR_DW_EMPTY, i), nb); // BC warps of this CTA and of each neighbour
      mbar_init(bar(BAR_AH_FULL, i), 8);   // BC warps
      mbar_init(bar(BAR_AH_EMPTY, i), 4);  // D warps
    }
    for (int w = 0; w < 4; ++w) {  // per pair (A warp w, D warp 12 + w), which share TMEM lanes and rows
      mbar_init(bar(BAR_XD, w), 1);  // D warp: its fields of the step's DW rows are written
      mbar_init(bar(BAR_YA, w), 1);  // A warp: the step's running sums are in TMEM
    }
    sm.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // halo rows without a neighbour are never written: zero padding
  for (int i = tid; i < 2 * 5 * 2 * R * SPAN; i += NT) {
    const int col = i % SPAN, rr = (i / SPAN) % (2 * R), f = (i / (SPAN * 2 * R)) % 5, bb = i / (SPAN * 2 * R * 5);
    if (!has_up) sm.dw[bb][rr][f][col] = 0.f;
    if (!has_dn) sm.dw[bb][TY + 2 * R + rr][f][col] = 0.f;
  }
  if (warp == 0) {
    const uint32_t dst = smem_addr(&sm.tmem_base);
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst), "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster.sync();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

  // The D group also boxes fields 3 and 4 (Stt, 2*Spt) of the A group's sums along W: A's W box is on
  // the loop that bounds a step (A writes plane s+2 once the column groups release plane s), the D group
  // idles while the column groups sweep.
  constexpr bool DASSIST = Geo<R>::DSUM_TMEM || ASSIST;
  constexpr int NFA = DASSIST ? 3 : 5;  // fields the A group boxes
  const float nf = a.n, nh = 0.5f * a.n, ndr = a.n * a.dr;
  double acc = 0.0;  // BC: loss partial
  // After a timed-out wait (a protocol error) every warp leaves its loops (warp-uniformly) without
  // arriving on any barrier or sending any copy again.
  bool a_aborted = false;

  // Segment walk shared by every role: the same (volume, tile, plane range) sequence and the same
  // global step counter s in every thread of the cluster.
  int64_t g0 = int64_t(blockIdx.y) * a.items_per_cluster;
  const int64_t g1 = min(g0 + a.items_per_cluster, a.total_items);
  uint32_t s = 0;
  while (g0 < g1) {
    if (role == 0 ? a_aborted : __any_sync(0xffffffffu, *abort_flag != 0)) break;
    Seg sg;
    {
      const int64_t item = g0 / Dout;
      const int64_t rem = g1 - item * Dout;
      sg.zs = a.z_begin + int(g0 - item * Dout);
      sg.ze = a.z_begin + int(rem < Dout ? rem : int64_t(Dout));
      g0 = item * Dout + (sg.ze - a.z_begin);
      const int tx = int(item % a.tiles_x);
      const int ty = int((item / a.tiles_x) % a.tiles_y);
      sg.b = item / (int64_t(a.tiles_x) * a.tiles_y);
      tile_geom(tx, W, SPAN, R, CW, sg.xb, sg.ox0, sg.ox1);
      tile_geom(ty, H, a.span_y, R, 1, sg.yb, sg.oy0, sg.oy1);
    }
    const int nsteps = sg.ze - sg.zs + 2 * R;
    const int c0 = sg.zs - R;
    const S* __restrict__ P = reinterpret_cast<const S*>(a.p) + sg.b * D * HW;
    const S* __restrict__ T = reinterpret_cast<const S*>(a.t) + sg.b * D * HW;
    const int64_t vofs = sg.b * D * HW;  // element offset of P and T from a.p and a.t
    // CW elements of the volume at element offset e (P/T relative); a checked build reads zeros outside
    auto gld = [&](const S* base, int64_t e, float4* o) {
      if (LNCC_IN(vofs + e, CW, a.n_in)) {
        Chunk<S, CW>::ld(base + e, o);
      } else {
#pragma unroll
        for (int h = 0; h < CW / 4; ++h) o[h] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    };

    // D warp's share of the W box of step st (fields 3 and 4 of the paired A warp's sums, same TMEM
    // lanes, same DW rows), once the buffer is free and the sums are complete; false after an abort.
    auto d_part = [&](uint32_t st, bool valid) -> bool {
      const int i = int(st & 1u);
      const int wq = warp & 3;
      mbar_wait(bar(BAR_DW_EMPTY, i), ((st >> 1) & 1u) ^ 1u, abort_flag);
      mbar_wait(bar(BAR_YA, wq), st & 1u, abort_flag);
      if (__any_sync(0xffffffffu, *abort_flag != 0)) return false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (valid) {
        const int yl = wq * 4 + (lane >> 3), q = lane & 7;
        const uint32_t tmA = sm.tmem_base + (uint32_t(32 * wq) << 16) + Geo<R>::TM_A;
        const uint32_t own = smem_addr(&sm.dw[i][2 * R + yl][0][0]);
        uint32_t choff[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) choff[j] = uint32_t(swz_chunk(4 * q + j) * 4);
        uint32_t ub[2][16];
        tm_ld16_issue(tmA + uint32_t(16 * 3), ub[0]);
        tm_wait_ld16(ub[0]);
#pragma unroll
        for (int f = 3; f < 5; ++f) {
          if (f == 3) tm_ld16_issue(tmA + uint32_t(16 * 4), ub[1]);
          float v[16];
#pragma unroll
          for (int m = 0; m < 16; ++m) v[m] = __uint_as_float(ub[f - 3][m]);
          wbox16<R>(v, q, [&](int j, float4 w4) { sts4(own + uint32_t(f * SPAN * 4) + choff[j], w4); });
          if (f == 3) tm_wait_ld16(ub[1]);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // for the halo bulk copy
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_cta(bar(BAR_XD, wq));
      return true;
    };
    auto plane_ok = [&](int it) { return c0 + it >= 0 && c0 + it < D; };

    if (role == 0) {
      // ===================================== A =========================================================
      const int yl = warp * 4 + (lane >> 3), q = lane & 7;
      const int Y = sg.yb + rank * TY + yl;
      const int X0 = sg.xb + VW * q;
      uint32_t cm = 0;  // valid CW-column chunks (W % CW == 0 and X0 % CW == 0: all or nothing)
#pragma unroll
      for (int j = 0; j < NCH; ++j)
        if (Y >= 0 && Y < H && X0 + CW * j >= 0 && X0 + CW * j < W) cm |= 1u << j;
      const int64_t roff = (cm ? int64_t(Y) * W + X0 : 0);
      const uint32_t tmA = sm.tmem_base + (uint32_t(32 * (warp & 3)) << 16) + Geo<R>::TM_A;
      uint32_t choff[4];  // byte offsets of this lane's four 4-column chunks in a swizzled row
#pragma unroll
      for (int j = 0; j < 4; ++j) choff[j] = uint32_t(swz_chunk(4 * q + j) * 4);
      const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
      // raw p, t of the plane entering (zi) and leaving (zo) the D window, this lane's 16 columns
      struct Raw {
        float4 pi[4], ti[4], po[4], to[4];
      };
      auto load_raw = [&](bool in_ok, int zi, bool out_ok, int zo, Raw& r) {
        constexpr int Q = CW / 4;
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
          const bool cj = (cm >> j) & 1u;
          if (in_ok && cj) {
            gld(P, zi * HW + roff + CW * j, &r.pi[Q * j]);
            gld(T, zi * HW + roff + CW * j, &r.ti[Q * j]);
          } else {
#pragma unroll
            for (int h = 0; h < Q; ++h) r.pi[Q * j + h] = r.ti[Q * j + h] = z4;
          }
          if (out_ok && cj) {
            gld(P, zo * HW + roff + CW * j, &r.po[Q * j]);
            gld(T, zo * HW + roff + CW * j, &r.to[Q * j]);
          } else {
#pragma unroll
            for (int h = 0; h < Q; ++h) r.po[Q * j + h] = r.to[Q * j + h] = z4;
          }
        }
      };
      // D update of the five running sums (TMEM, 16 columns per field) with a Raw pair of planes.
      // Fields in an order that lets the raw registers die early: 2*Spt, Spp, Sp, Stt, St.
      auto dsum_update = [&](const Raw& r) {
        float2 dp[8], sp[8], dt[8], st[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          dp[2 * j] = sub2(make_float2(r.pi[j].x, r.pi[j].y), make_float2(r.po[j].x, r.po[j].y));
          dp[2 * j + 1] = sub2(make_float2(r.pi[j].z, r.pi[j].w), make_float2(r.po[j].z, r.po[j].w));
          sp[2 * j] = add2(make_float2(r.pi[j].x, r.pi[j].y), make_float2(r.po[j].x, r.po[j].y));
          sp[2 * j + 1] = add2(make_float2(r.pi[j].z, r.pi[j].w), make_float2(r.po[j].z, r.po[j].w));
          dt[2 * j] = sub2(make_float2(r.ti[j].x, r.ti[j].y), make_float2(r.to[j].x, r.to[j].y));
          dt[2 * j + 1] = sub2(make_float2(r.ti[j].z, r.ti[j].w), make_float2(r.to[j].z, r.to[j].w));
          st[2 * j] = add2(make_float2(r.ti[j].x, r.ti[j].y), make_float2(r.to[j].x, r.to[j].y));
          st[2 * j + 1] = add2(make_float2(r.ti[j].z, r.ti[j].w), make_float2(r.to[j].z, r.to[j].w));
        }
        tm_wait_st();
#pragma unroll
        for (int fi = 0; fi < 5; ++fi) {
          const int f = fi == 0 ? 4 : fi == 1 ? 2 : fi == 2 ? 0 : fi == 3 ? 3 : 1;
          float v[16];
          tm_ld16(tmA + uint32_t(16 * f), v);
#pragma unroll
          for (int m = 0; m < 8; ++m) {
            float2 x2 = make_float2(v[2 * m], v[2 * m + 1]);
            if (f == 0) x2 = add2(x2, dp[m]);
            else if (f == 1) x2 = add2(x2, dt[m]);
            else if (f == 2) x2 = fma2(dp[m], sp[m], x2);
            else if (f == 3) x2 = fma2(dt[m], st[m], x2);
            else x2 = fma2(dp[m], st[m], fma2(sp[m], dt[m], x2));
            v[2 * m] = x2.x;
            v[2 * m + 1] = x2.y;
          }
          tm_st16(tmA + uint32_t(16 * f), v);
        }
      };
      // the warm-up below loads its raw planes one after another: ask for all of them in L2 first
      if (cm) {
        for (int z = c0 - R; z <= c0 + R; ++z) {
          if (z < 0 || z >= D) continue;
#pragma unroll
          for (int j = 0; j < NCH; ++j) {
            if (!((cm >> j) & 1u)) continue;
            asm volatile("prefetch.global.L2 [%0];" ::"l"(P + z * HW + roff + CW * j));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(T + z * HW + roff + CW * j));
          }
        }
      }
      // zero the sums, then warm up over raw planes [c0 - R, c0 + R)
      tm_wait_st();
      {
        const uint32_t zr[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll
        for (int f = 0; f < 10; ++f) tm_st8(tmA + uint32_t(8 * f), zr);
      }
      for (int z = c0 - R; z < c0 + R; ++z) {
        if (z < 0 || z >= D) continue;
        Raw r;
        load_raw(true, z, false, 0, r);
        dsum_update(r);
      }
      {
        Raw r;  // step 0: add raw plane c0 + R
        load_raw(c0 + R < D, c0 + R, false, 0, r);
        dsum_update(r);
      }
      // the sums of a step are complete: the paired D warp may box its fields
      auto sums_ready = [&]() {
        if constexpr (DASSIST) {
          tm_wait_st();
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive_cta(bar(BAR_YA, warp));
        }
      };
      sums_ready();
      // halo rows sent to the neighbours by bulk copy, per field: my first 2R rows go to the CTA above
      // (its rows [TY + 2R, TY + 4R)), my last 2R rows to the CTA below (its rows [0, 2R))
      constexpr uint32_t kHaloBytes = 2 * R * 5 * SPAN * 4;  // 2R rows x 5 fields
      const uint32_t rx_bytes = kHaloBytes * ((has_up ? 1u : 0u) + (has_dn ? 1u : 0u));
      for (int it = 0; it < nsteps; ++it, ++s) {
        const int c = c0 + it;
        const bool cvalid = c >= 0 && c < D;
        const int i = int(s & 1u);
        // the next step's raw planes are loaded now and used after this step's W box
        const bool more = it + 1 < nsteps;
        const int zi = c + 1 + R, zo = c - R;
        Raw r;
        load_raw(more && zi < D, zi, more && zo >= 0, zo, r);
        mbar_wait(bar(BAR_DW_EMPTY, i), ((s >> 1) & 1u) ^ 1u, abort_flag);
        if (__any_sync(0xffffffffu, *abort_flag != 0)) {
          a_aborted = true;
          break;
        }
        if (cvalid) {
          // W box of each field -> the CTA's own DW rows
          tm_wait_st();
          const uint32_t own = smem_addr(&sm.dw[i][2 * R + yl][0][0]);
          // the next field's TMEM load is in flight while this field is boxed
          uint32_t ub[2][16];
          tm_ld16_issue(tmA, ub[0]);
          tm_wait_ld16(ub[0]);
#pragma unroll
          for (int f = 0; f < NFA; ++f) {
            if (f + 1 < NFA) tm_ld16_issue(tmA + uint32_t(16 * (f + 1)), ub[(f + 1) & 1]);
            float v[16];
#pragma unroll
            for (int m = 0; m < 16; ++m) v[m] = __uint_as_float(ub[f & 1][m]);
            wbox16<R>(v, q, [&](int j, float4 w4) { sts4(own + uint32_t(f * SPAN * 4) + choff[j], w4); });
            if (f + 1 < NFA) tm_wait_ld16(ub[(f + 1) & 1]);
          }
        }
        // make this warp's rows visible to the bulk-copy (async) proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if constexpr (DASSIST) {  // the paired D warp's fields of these rows
          mbar_wait(bar(BAR_XD, warp), s & 1u, abort_flag);
          if (__any_sync(0xffffffffu, *abort_flag != 0)) {
            a_aborted = true;
            break;
          }
        }
        if (lane == 0) {
          // warp 0 also announces the halo bytes the neighbours send into this CTA for this step
          if (warp == 0) mbar_arrive_expect_tx(bar(BAR_DW_FULL, i), rx_bytes);
          else mbar_arrive_cta(bar(BAR_DW_FULL, i));
          // Halo rows to the neighbours, each warp its own rows (all five fields of a row are
          // contiguous): the CTA's first 2R rows become the CTA above's rows [TY + 2R, TY + 4R), its
          // last 2R rows the CTA below's rows [0, 2R). Sent on every step, also for planes outside the
          // volume (whose rows nobody reads): a neighbour's column groups can then never run two steps
          // ahead of this CTA, because their step-s+2 input includes these copies, which are issued
          // only after this CTA's step-s buffer was released.
          const int r0 = 4 * warp, r1 = 4 * warp + 4;  // this warp's rows
          constexpr uint32_t kRowBytes = 5 * SPAN * 4;
          if (has_up && r0 < 2 * R && LNCC_IN_SMEM(smem_addr(&sm.dw[i][TY + 2 * R + r0][0][0]), uint32_t((r1 < 2 * R ? r1 : 2 * R) - r0) * kRowBytes)) {
            const int e1 = r1 < 2 * R ? r1 : 2 * R;
            bulk_copy_to_peer(mapa_rank(smem_addr(&sm.dw[i][TY + 2 * R + r0][0][0]), uint32_t(rank - 1)),
                              smem_addr(&sm.dw[i][2 * R + r0][0][0]), uint32_t(e1 - r0) * kRowBytes,
                              mapa_rank(bar(BAR_DW_FULL, i), uint32_t(rank - 1)));
          }
          if (has_dn && r1 > TY - 2 * R &&
              LNCC_IN_SMEM(smem_addr(&sm.dw[i][(r0 > TY - 2 * R ? r0 : TY - 2 * R) - (TY - 2 * R)][0][0]),
                           uint32_t(r1 - (r0 > TY - 2 * R ? r0 : TY - 2 * R)) * kRowBytes)) {
            const int b0 = r0 > TY - 2 * R ? r0 : TY - 2 * R;
            bulk_copy_to_peer(mapa_rank(smem_addr(&sm.dw[i][b0 - (TY - 2 * R)][0][0]), uint32_t(rank + 1)),
                              smem_addr(&sm.dw[i][2 * R + b0][0][0]), uint32_t(r1 - b0) * kRowBytes,
                              mapa_rank(bar(BAR_DW_FULL, i), uint32_t(rank + 1)));
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          reg_fence(r.pi[j]);
          reg_fence(r.ti[j]);
          reg_fence(r.po[j]);
          reg_fence(r.to[j]);
        }
        if (more) {
          // the D warp has read this step's fields 3 and 4 (its arrival came after its TMEM loads)
          if constexpr (DASSIST) asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          dsum_update(r);
          sums_ready();
        }
      }
    } else if (role == 1 || role == 2) {
      // ===================================== BC ========================================================
      // two threads per column: half h sweeps DW rows [8h, 8h + 8 + 4R) and produces AH rows [8h, 8h + 8)
      constexpr int HR = TY / 2;           // AH rows per half
      constexpr int ERH = HR + 4 * R;      // DW rows per half
      const int h = role - 1;
      const int x = tid - 128 * role;
      const int px = swz(x);
      const int X = sg.xb + x;
      const bool col_valid = X >= 0 && X < W;
      const bool col_own = X >= sg.ox0 && X < sg.ox1;
      // bit k: stat row ys = HR*h - R + k lies in the volume (vmask) / is an output row of this half
      // (omask; each half counts the cc of its own HR rows only)
      uint32_t vmask = 0, omask = 0;
      {
        const int ybase = sg.yb + rank * TY;  // global row of band row 0
#pragma unroll
        for (int k = 0; k < HR + 2 * R; ++k) {
          const int ys = HR * h - R + k;
          const int Yg = ybase + ys;
          if (col_valid && Yg >= 0 && Yg < H) vmask |= 1u << k;
          if (ys >= HR * h && ys < HR * h + HR && col_own && Yg >= sg.oy0 && Yg < sg.oy1) omask |= 1u << k;
        }
      }
      const float2 nneg2 = make_float2(-nf, -nf);
      const float2 ndr2 = make_float2(ndr, ndr);
      for (int it = 0; it < nsteps; ++it, ++s) {
        const int i = int(s & 1u);
        const uint32_t ph = (s >> 1) & 1u;
        const int c = c0 + it;
        const bool cvalid = c >= 0 && c < D;
        const uint32_t om_step = (it >= R && it < nsteps - R) ? omask : 0u;  // plane c is an output plane
        mbar_wait(bar(BAR_DW_FULL, i), ph, abort_flag);
        if (GRAD) mbar_wait(bar(BAR_AH_EMPTY, i), ph ^ 1u, abort_flag);
        if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
        if (cvalid) {
          const float* dwp = &sm.dw[i][HR * h][0][px];
          // running H sums: (Sp, St) and -n * (Spp, Stt) as f32x2 pairs, 2*Spt alone; windows of the
          // last K rows
          float2 win01[K], win23[K];
          float win4[K];
          float2 s01 = make_float2(0.f, 0.f), s23 = make_float2(0.f, 0.f);
          float s4 = 0.f;
          float2 awab[K];
          float awc[K];
          float2 aab = make_float2(0.f, 0.f);
          float ac = 0.f;
          float cc_acc = 0.f;
#pragma unroll
          for (int e = 0; e < ERH; ++e) {
            auto lds = [&](int off) -> float { return LNCC_IN_SMEM_PTR(dwp + off, 4) ? dwp[off] : 0.f; };
            const float2 v01 = make_float2(lds((e * 5 + 0) * SPAN), lds((e * 5 + 1) * SPAN));
            const float2 v23 = make_float2(lds((e * 5 + 2) * SPAN), lds((e * 5 + 3) * SPAN));
            const float v4 = lds((e * 5 + 4) * SPAN);
            if (e >= K) {
              s01 = add2(s01, sub2(v01, win01[e % K]));
              s23 = fma2(nneg2, sub2(v23, win23[e % K]), s23);
              s4 += v4 - win4[e % K];
            } else {
              s01 = add2(s01, v01);
              s23 = fma2(nneg2, v23, s23);
              s4 += v4;
            }
            win01[e % K] = v01;
            win23[e % K] = v23;
            win4[e % K] = v4;
            if (e >= 2 * R) {
              const int k = e - 2 * R;  // stat row HR*h - R + k
              const float Sp = s01.x, St = s01.y;
              // (-VP', -VT') = (Sp^2 - n*Spp, St^2 - n*Stt); VP = max(n*Spp - Sp^2, 0) + n*dr, VT alike
              const float2 mv = fma2(s01, s01, s23);
              const float2 vpt = sub2(ndr2, make_float2(fminf(mv.x, 0.f), fminf(mv.y, 0.f)));
              const float VP = vpt.x, VT = vpt.y;
              const float Xc = fmaf(nh, s4, -(Sp * St));
              float rden;
              asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(rden) : "f"(VP * VT));
              const float wq = Xc * rden;
              const float cc = Xc * wq;
              if ((om_step >> k) & 1u) {
                float ccl;  // min(cc, 1), NaN kept (the reference does not mask NaN)
                asm("min.NaN.f32 %0, %1, %2;" : "=f"(ccl) : "f"(cc), "f"(1.f));
                cc_acc += ccl;
              }
              if (GRAD) {
                // NaN and cc >= 1: zero adjoints (lncc3d.cu:100-107); rows outside the volume: zero
                const bool live = ((vmask >> k) & 1u) && (cc < 1.f);
                const float wv = wq * VT;
                float2 ab = __fmul2_rn(make_float2(wq, wq), make_float2(fmaf(-wv, Sp, St), wv));
                ab = live ? ab : make_float2(0.f, 0.f);
                const float cq = live ? wq : 0.f;
                if (k >= K) {
                  aab = add2(aab, sub2(ab, awab[k % K]));
                  ac += cq - awc[k % K];
                } else {
                  aab = add2(aab, ab);
                  ac += cq;
                }
                awab[k % K] = ab;
                awc[k % K] = cq;
                if (k >= 2 * R) {
                  const int yo = HR * h + k - 2 * R;
                  if (LNCC_IN_SMEM_PTR(&sm.ah[i][0][yo][px], 4)) sm.ah[i][0][yo][px] = aab.x;
                  if (LNCC_IN_SMEM_PTR(&sm.ah[i][1][yo][px], 4)) sm.ah[i][1][yo][px] = aab.y;
                  if (LNCC_IN_SMEM_PTR(&sm.ah[i][2][yo][px], 4)) sm.ah[i][2][yo][px] = ac;
                }
              }
            }
          }
          acc += double(cc_acc);
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_cta(bar(BAR_DW_EMPTY, i));
          if (has_up) mbar_arrive_remote_relaxed(bar(BAR_DW_EMPTY, i), uint32_t(rank - 1));
          if (has_dn) mbar_arrive_remote_relaxed(bar(BAR_DW_EMPTY, i), uint32_t(rank + 1));
          if (GRAD) mbar_arrive_cta(bar(BAR_AH_FULL, i));
        }
      }
    } else if (GRAD) {
      // ===================================== D =========================================================
      const int yl = (warp - 12) * 4 + (lane >> 3), q = lane & 7;
      const int Y = sg.yb + rank * TY + yl;
      const int X0 = sg.xb + VW * q;
      uint32_t om = 0;  // output CW-column chunks
      if (Y >= sg.oy0 && Y < sg.oy1) {
#pragma unroll
        for (int j = 0; j < NCH; ++j)
          if (X0 + CW * j >= sg.ox0 && X0 + CW * j < sg.ox1) om |= 1u << j;
      }
      const int64_t roff = om ? int64_t(Y) * W + X0 : 0;
      S* __restrict__ G = reinterpret_cast<S*>(a.g) + sg.b * int64_t(a.g_planes) * HW;
      const uint32_t tm = sm.tmem_base + (uint32_t(32 * (warp & 3)) << 16);
      const float gs = 2.f * a.gscale * (a.gscale_dev ? __ldg(a.gscale_dev) : 1.f);
      const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
      // AH row of field f for this lane -> W box; emit(j, float4) gets the boxed chunk j
      auto box_ah = [&](int i, int f, auto&& emit) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float* ahp = &sm.ah[i][f][yl][swz_chunk(4 * q + j)];
          const float4 w4 = LNCC_IN_SMEM_PTR(ahp, 16) ? *reinterpret_cast<const float4*>(ahp) : make_float4(0.f, 0.f, 0.f, 0.f);
          v[4 * j] = w4.x;
          v[4 * j + 1] = w4.y;
          v[4 * j + 2] = w4.z;
          v[4 * j + 3] = w4.w;
        }
        if (f == 2) {  // every AH value this warp needs is in registers
          __syncwarp();
          if (lane == 0) mbar_arrive_cta(bar(BAR_AH_EMPTY, i));
        }
        wbox16<R>(v, q, emit);
      };
      auto release_ah = [&](int i) {
        __syncwarp();
        if (lane == 0) mbar_arrive_cta(bar(BAR_AH_EMPTY, i));
      };
      // grad = gs * (n*t*Sc - n*p*Sb - Sa) for chunk j (gs carries the 2 and the loss scale)
      auto grad4 = [&](float4 p4, float4 t4, const float* sa, const float* sb, const float* sc) {
        const float pq[4] = {p4.x, p4.y, p4.z, p4.w}, tq[4] = {t4.x, t4.y, t4.z, t4.w};
        float g4[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) g4[m] = gs * fmaf(nf, fmaf(tq[m], sc[m], -pq[m] * sb[m]), -sa[m]);
        return make_float4(g4[0], g4[1], g4[2], g4[3]);
      };
      int slot = 0;
      if constexpr (Geo<R>::DSUM_TMEM) {
        // running sums in TMEM; p, t of the output plane are loaded at the start of the step
        const uint32_t tsum = tm + Geo<R>::TM_DSUM;
        // the W-box share of the segment's first two steps, then of step s + 2 before step s's adjoints
        if (!d_part(s, plane_ok(0)) || !d_part(s + 1, plane_ok(1))) break;
        for (int it = 0; it < nsteps; ++it, ++s) {
          if (it + 2 < nsteps && !d_part(s + 2, plane_ok(it + 2))) break;
          const int c = c0 + it;
          const bool cvalid = c >= 0 && c < D;
          const int o = c - R;
          const bool out_ok = it >= 2 * R && om != 0;
          const int i = int(s & 1u);
          float4 pv[4], tv[4];
#pragma unroll
          for (int j = 0; j < NCH; ++j) {
            constexpr int Q = CW / 4;
            if (out_ok && ((om >> j) & 1u)) {
              gld(P, o * HW + roff + CW * j, &pv[Q * j]);
              gld(T, o * HW + roff + CW * j, &tv[Q * j]);
            } else {
#pragma unroll
              for (int h = 0; h < Q; ++h) pv[Q * j + h] = tv[Q * j + h] = z4;
            }
          }
          tm_wait_st();
          mbar_wait(bar(BAR_AH_FULL, i), (s >> 1) & 1u, abort_flag);
          if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
#pragma unroll
          for (int f = 0; f < 3; ++f) {
            const uint32_t ring = tm + Geo<R>::TM_RING + uint32_t(48 * slot + 16 * f);
            uint32_t uo[16], us[16];
            if (it >= K) {
              tm_ld16_issue(ring, uo);  // the boxed plane leaving the D window
            } else {
#pragma unroll
              for (int m = 0; m < 16; ++m) uo[m] = 0u;
            }
            if (it > 0) {
              tm_ld16_issue(tsum + uint32_t(16 * f), us);
            } else {
#pragma unroll
              for (int m = 0; m < 16; ++m) us[m] = 0u;
            }
            // one wait covers both loads; the second names the other registers so that their uses
            // follow it
            tm_wait_ld16(us);
            tm_wait_ld16(uo);
            float old[16], sum[16];
#pragma unroll
            for (int m = 0; m < 16; ++m) {
              old[m] = __uint_as_float(uo[m]);
              sum[m] = __uint_as_float(us[m]);
            }
            if (cvalid) {
              box_ah(i, f, [&](int j, float4 w4) {
                const float2 lo = add2(make_float2(sum[4 * j], sum[4 * j + 1]),
                                       sub2(make_float2(w4.x, w4.y), make_float2(old[4 * j], old[4 * j + 1])));
                const float2 hi = add2(make_float2(sum[4 * j + 2], sum[4 * j + 3]),
                                       sub2(make_float2(w4.z, w4.w), make_float2(old[4 * j + 2], old[4 * j + 3])));
                sum[4 * j] = lo.x;
                sum[4 * j + 1] = lo.y;
                sum[4 * j + 2] = hi.x;
                sum[4 * j + 3] = hi.y;
                tm_st4(ring + uint32_t(4 * j), w4);
              });
            } else {
              if (f == 2) release_ah(i);
#pragma unroll
              for (int m = 0; m < 16; ++m) sum[m] -= old[m];
#pragma unroll
              for (int j = 0; j < 4; ++j) tm_st4(ring + uint32_t(4 * j), z4);
            }
            tm_st16(tsum + uint32_t(16 * f), sum);
          }
          if (it >= 2 * R) {  // warp-uniform: the TMEM loads below are warp-collective
            tm_wait_st();
            float sa[16], sb[16], sc[16];
            {
              uint32_t ua[16], ub[16], uc[16];
              tm_ld16_issue(tsum, ua);
              tm_ld16_issue(tsum + 16u, ub);
              tm_ld16_issue(tsum + 32u, uc);
              tm_wait_ld16(ua);
              tm_wait_ld16(ub);
              tm_wait_ld16(uc);
#pragma unroll
              for (int m = 0; m < 16; ++m) {
                sa[m] = __uint_as_float(ua[m]);
                sb[m] = __uint_as_float(ub[m]);
                sc[m] = __uint_as_float(uc[m]);
              }
            }
            if (out_ok) {
              S* gp = G + int64_t(o - a.z_begin) * HW + roff;
              constexpr int Q = CW / 4;
#pragma unroll
              for (int j = 0; j < NCH; ++j) {
                if (!((om >> j) & 1u)) continue;
                float4 g4[Q];
#pragma unroll
                for (int h = 0; h < Q; ++h) {
                  const int c4 = Q * j + h;
                  g4[h] = grad4(pv[c4], tv[c4], sa + 4 * c4, sb + 4 * c4, sc + 4 * c4);
                }
                if (LNCC_IN((gp - reinterpret_cast<S*>(a.g)) + CW * j, CW, a.n_g)) Chunk<S, CW>::st(gp + CW * j, g4);
              }
            }
          }
          slot = (slot + 1 == K) ? 0 : slot + 1;
        }
      } else {
        // running sums in registers (k = 9: TMEM holds the ring and the A group's sums)
        float sum[3][16];
#pragma unroll
        for (int f = 0; f < 3; ++f)
#pragma unroll
          for (int m = 0; m < 16; ++m) sum[f][m] = 0.f;
        if constexpr (DASSIST) {  // the W-box share of the segment's first two steps
          if (!d_part(s, plane_ok(0)) || !d_part(s + 1, plane_ok(1))) break;
        }
        for (int it = 0; it < nsteps; ++it, ++s) {
          if constexpr (DASSIST) {  // and of step s + 2 before step s's adjoints
            if (it + 2 < nsteps && !d_part(s + 2, plane_ok(it + 2))) break;
          }
          const int c = c0 + it;
          const bool cvalid = c >= 0 && c < D;
          const int o = c - R;
          const bool out_ok = it >= 2 * R && om != 0;
          const int i = int(s & 1u);
          tm_wait_st();
          mbar_wait(bar(BAR_AH_FULL, i), (s >> 1) & 1u, abort_flag);
          if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
#pragma unroll
          for (int f = 0; f < 3; ++f) {
            const uint32_t ring = tm + Geo<R>::TM_RING + uint32_t(48 * slot + 16 * f);
            float old[16];
            if (it >= K) tm_ld16(ring, old);
            else {
#pragma unroll
              for (int m = 0; m < 16; ++m) old[m] = 0.f;
            }
            if (cvalid) {
              box_ah(i, f, [&](int j, float4 w4) {
                sum[f][4 * j] += w4.x - old[4 * j];
                sum[f][4 * j + 1] += w4.y - old[4 * j + 1];
                sum[f][4 * j + 2] += w4.z - old[4 * j + 2];
                sum[f][4 * j + 3] += w4.w - old[4 * j + 3];
                tm_st4(ring + uint32_t(4 * j), w4);
              });
            } else {
              if (f == 2) release_ah(i);
#pragma unroll
              for (int m = 0; m < 16; ++m) sum[f][m] -= old[m];
#pragma unroll
              for (int j = 0; j < 4; ++j) tm_st4(ring + uint32_t(4 * j), z4);
            }
          }
          if (out_ok) {
            S* gp = G + int64_t(o - a.z_begin) * HW + roff;
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
              if (!((om >> j) & 1u)) continue;
              constexpr int Q = CW / 4;
              float4 p4[Q], t4[Q], g4[Q];
              gld(P, o * HW + roff + CW * j, p4);
              gld(T, o * HW + roff + CW * j, t4);
#pragma unroll
              for (int h = 0; h < Q; ++h) {
                const int c4 = Q * j + h;
                g4[h] = grad4(p4[h], t4[h], sum[0] + 4 * c4, sum[1] + 4 * c4, sum[2] + 4 * c4);
              }
              if (LNCC_IN((gp - reinterpret_cast<S*>(a.g)) + CW * j, CW, a.n_g)) Chunk<S, CW>::st(gp + CW * j, g4);
            }
          }
          slot = (slot + 1 == K) ? 0 : slot + 1;
        }
      }
    } else {
      // loss only: the D group's work is its share of the W box
      if constexpr (DASSIST) {
        if (!d_part(s, plane_ok(0)) || !d_part(s + 1, plane_ok(1))) break;
        for (int it = 0; it < nsteps; ++it, ++s)
          if (it + 2 < nsteps && !d_part(s + 2, plane_ok(it + 2))) break;
      } else {
        s += uint32_t(nsteps);
      }
    }
  }

  // ---- teardown: nobody leaves while a neighbour can still write into its shared memory ---------------
  if (role == 1 || role == 2) {
    double d = acc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) d += __shfl_down_sync(0xffffffffu, d, o);
    if (lane == 0) sm.red[warp - 4] = d;
  }
  if (role == 0 || (GRAD && role == 3)) tm_wait_st();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster.sync();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(sm.tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
  if (tid == 0) {
    double tot = 0.0;
    for (int w = 0; w < 8; ++w) tot += sm.red[w];
    if (sm.abort_flag) {  // a wait timed out: NaN partial, and the abort word for callers without a loss
      tot = __longlong_as_double(0x7ff8000000000000ll);
      if (a.abort_word) atomicOr(a.abort_word, 1u);
    }
    const int64_t pi = int64_t(blockIdx.y) * gridDim.x + blockIdx.x;
    if (LNCC_IN(pi, 1, a.n_parts)) a.partials[pi] = tot;
  }
}

// Self-test of the bounded wait and of the abort record: one warp waits on a barrier that nothing
// arrives at, with a limit of `limit_ns`; the wait gives up, and the warp records the abort in
// `word` exactly as the fused kernel's teardown does. No cluster, bulk copy or TMEM is involved.
__global__ void __launch_bounds__(32, 1) wait_timeout_selftest_kernel(unsigned* word, unsigned long long limit_ns) {
  __shared__ unsigned long long bar;
  __shared__ int abort_flag;
  const uint32_t b = smem_addr(&bar);
  if (threadIdx.x == 0) {
    *word = 0u;
    abort_flag = 0;
    mbar_init(b, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  mbar_wait_slow(b, 0u, &abort_flag, limit_ns);  // phase 0 never completes
  __syncwarp();
  if (threadIdx.x == 0 && abort_flag) atomicOr(word, 1u);
}

}  // namespace ws
}  // namespace lncc
