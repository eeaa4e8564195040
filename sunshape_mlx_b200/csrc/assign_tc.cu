// Nearest-centroid assignment on the 5th-generation tensor cores (tcgen05),
// exact with respect to the reference's float32 CPU arithmetic.
//
// The reference picks, per key row and block b, argmin_c of a float32 distance
// evaluated in NumPy order (codec.py:497-499 direct form; codec.py:88-91
// expanded form inside k-means). Here the distance is screened as a GEMM and
// only near ties are re-evaluated exactly:
//
//   screen  V(c) = ||c||^2 - 2 k.c   (one M=128 x N=k x K=Kt tcgen05 MMA chain
//                                     per (128-row tile, block), fp32 in TMEM)
//   A row   [-2 kh | -2 kh | -2 kl | 1, 1, 0...]      (fp16, Kt = 16*ceil((3bd+2)/16))
//   B row   [  ch  |  cl   |  ch   | csq_h, csq_l, 0...]
//
// with x = xh + xl the fp16 hi/lo split of a float32 value, after scaling the
// block by a power of two so that its largest centroid component is in [1, 2).
// The epilogue (one thread per row) reads the row's V once from TMEM and
// keeps the minima of two partitions of the columns (by high and by low
// nibble of the centroid index; three-input mins, ALU pipe). A single group
// below s1 + T in each partition means no other centroid lies within T of
// the minimum s1 (two distinct indices differ in a nibble), and the two
// groups give the winner's index. Error analysis (u = 2^-24,
// S = ||k||^2 + max_c ||c||^2, all in scaled units, per value; a comparison
// of two values doubles each term):
//   |reference distance - exact real distance| <= 2^-19 S (either mode),
//   |V - (exact distance - ||k||^2)|         <= 2^-17 S (fp16 splits 2^-22,
//        the dropped kl*cl term 2^-22, the csq split 2^-21, fp16 subnormals
//        2^-20, and the fp32 accumulation of <= 26 exact products with one
//        rounding or truncation of 2^-23 relative per addition, 2^-17.4).
// Doubled and summed that is < 2^-15.5 S, and T = 2^-14 S. So when the count
// is 1 no other centroid can have a reference distance <= the winner's, and
// the winner is the reference's argmin. Rows
// where that gap test fails (or whose values are not finite, or whose scaled
// key does not fit fp16) are re-scored exactly by the whole warp in the
// reference order, ties to the lowest index (np.argmin, kernels.py:1020).
//
// CTA roles (384 threads, one CTA per SM, persistent over 128-row tiles of
// one row group each):
//   warps 0-7   epilogue: warp w reads TMEM lanes 32*(w%4)..+31; warps 0-3
//               take even sequence steps (TMEM buffer 0), warps 4-7 odd ones
//   warp 8      TMEM allocation; lane 0 of warps 0 and 4 issues its group's
//               MMAs, whose completion frees the A slot and fills the TMEM
//               buffer
//   warps 9-10  producers: gather each row's permuted block from the staged
//               key tile into the A operand (canonical no-swizzle K-major
//               layout) and hand the scaled key norms to the epilogue
//   warp 11     loader: stages key tiles (16-byte cp.async copies into a
//               padded shared-memory tile) as far ahead as the ring allows
// A sequence step is one (tile, block) pair; blocks of a CTA are a contiguous
// group of the codec's blocks whose B operands stay resident in shared memory.
#include <atomic>

#include "common.cuh"
#include "vq_math.cuh"

namespace ss {

__device__ unsigned int g_assign_status = 0;  // sticky: 1 = a pipeline wait gave up

namespace {

constexpr int kTcRows = 128;            // MMA M (rows per tile)
constexpr int kKnRing = 4;              // key-norm hand-off ring (producers -> epilogue)
constexpr int kTcMmaWarp = 8;
constexpr int kTcProdWarp0 = 9;
constexpr int kTcProdThreads = 64;
constexpr int kTcLoadWarp = kTcProdWarp0 + kTcProdThreads / 32;    // 11
constexpr int kTcThreads = (kTcLoadWarp + 1) * 32;                  // 384
constexpr uint64_t kTcWaitNs = 2000000000ull;                      // 2 s per wait
constexpr float kTieRel = 1.0f / 16384.0f;                          // 2^-14

struct TcParams {
  const void* keys;
  int key_dtype, es;
  int64_t n_groups, rpg, kgs, krs;
  int d, nb, k, bd, kt;
  const int32_t* perm;
  const float* cents;
  const uint8_t* heavy;
  uint8_t* out_idx;
  int64_t igs, irs;
  uint16_t* out_heavy;
  int64_t hgs, hrs;
  float* out_pt;
  int dist_mode;
  int n_grp, gsize;       // block groups and blocks per group
  int slots;              // A ring depth
  int nstage;             // staged key tiles in flight (2 or 3)
  int64_t tpg, n_tiles;   // 128-row tiles per group, total tiles
  uint64_t wait_ns;       // bound of every pipeline wait
  int64_t skip_tile;      // test hook: tile the loader never stages (-1: none)
  int* sink;              // process error sink (host word) or null
  // dynamic shared-memory offsets (bytes, from the 1024-aligned base)
  uint32_t off_b, off_a, off_stage, off_cf, off_misc, stage_bytes, stage_stride;
};

// ---- tcgen05 wrappers -------------------------------------------------------
__device__ __forceinline__ void tc_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, fp16 inputs, fp32 accumulator.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives (once) on an mbarrier when all earlier MMAs of this thread are done.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
        "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
        "=r"(v[31])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor, canonical K-major layout without swizzle:
// 8-row x 16-byte core matrices, `lbo` bytes between K-adjacent core
// matrices and `sbo` bytes between 8-row groups.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  return d;                // base offset 0, layout type 0 (no swizzle)
}
// Instruction descriptor: fp16 A/B, fp32 D, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t instr_desc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
}

template <int BD>
struct TcShape {
  static constexpr int kKt = ((3 * BD + 2) + 15) / 16 * 16;  // K of the MMA chain
};


__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Byte offset of element (row, kel) in a canonical K-major tile with kt columns.
__device__ __forceinline__ uint32_t kmaj_off(int row, int kel, int kt) {
  return (uint32_t)((row >> 3) * (kt * 16) + (kel >> 3) * 128 + (row & 7) * 16 + (kel & 7) * 2);
}

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                        const TcParams& p) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (global_ns() - t0 > p.wait_ns) {
      if (!*abort) report_wait_failure(nullptr, p.sink, 16);
      *abort = 1;
      atomicOr(&g_assign_status, 1u);
      return false;
    }
  }
}

// Exact re-score of one (row, block) by the whole warp, reference order,
// sequential '<' semantics of the reference loop: the first index whose
// distance is below every earlier one; a NaN distance at index 0 keeps 0.
// kk: the row's permuted block values (float32, unscaled); cb: the block's
// float32 centroids in shared memory.
template <int BD>
__device__ int exact_rescan(const float (&kk)[BD], const float* cb, int k, int dist_mode,
                            int lane) {
  float best = __int_as_float(0x7f800000);
  int bi = 0x7fffffff;
  float d0 = 0.f;
  for (int c = lane; c < k; c += 32) {
    float cv[BD];
#pragma unroll
    for (int q = 0; q < BD; q += 4) {
      const float4 f = *reinterpret_cast<const float4*>(cb + c * BD + q);
      cv[q] = f.x; cv[q + 1] = f.y; cv[q + 2] = f.z; cv[q + 3] = f.w;
    }
    const float dd = dist_mode == 0 ? dist_direct<BD>(kk, cv) : dist_expanded<BD>(kk, cv);
    if (c == 0) d0 = dd;
    if (dd < best) { best = dd; bi = c; }
  }
  d0 = __shfl_sync(0xffffffffu, d0, 0);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob < best || (ob == best && oi < bi)) { best = ob; bi = oi; }
  }
  if (d0 != d0 || bi == 0x7fffffff) return 0;
  return bi;
}

// Element at byte column cb of tile row `row` in a staged key tile (rows
// padded by 16 bytes so a column read by 32 consecutive rows hits 8 banks).
__device__ __forceinline__ float stage_val(const uint8_t* st, uint32_t stride, int row, int cb,
                                           int dt) {
  const uint8_t* q = st + row * stride + cb;
  if (dt == SS_F32) return *reinterpret_cast<const float*>(q);
  const uint16_t u = *reinterpret_cast<const uint16_t*>(q);
  return dt == SS_F16 ? h2f(u) : bf2f(u);
}

template <int BD>
__global__ void __launch_bounds__(kTcThreads, 1)
    vq_assign_tc_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* s_b = smem + p.off_b;
  uint8_t* s_a = smem + p.off_a;
  uint8_t* s_stage = smem + p.off_stage;
  uint8_t* misc = smem + p.off_misc;
  float* s_cf = reinterpret_cast<float*>(smem + p.off_cf);         // [gsize][k][BD] f32
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc);              // 2*slots + 10 + 16 (<= 32)
  int16_t* s_pcol = reinterpret_cast<int16_t*>(misc + 256);        // [d] permuted column bytes
  float* s_scale = reinterpret_cast<float*>(misc + 256 + 1024);    // [gsize]
  float* s_cmax = s_scale + 32;  // [gsize] max scaled ||c||^2
  float* s_slo = s_cmax + 32;    // [gsize] scaled S below which fp32 distances may underflow
  float* s_shi = s_slo + 32;     // [gsize] scaled S above which they may overflow
  uint8_t* s_heavy = reinterpret_cast<uint8_t*>(s_shi + 32);        // [nb]
  uint8_t* s_hpos = s_heavy + 128;                                  // [nb]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(s_hpos + 128);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  uint64_t* a_full = bars;                 // [slots] producers -> MMA (64 arrivals)
  uint64_t* a_empty = bars + p.slots;      // [slots] MMA commit -> producers
  uint64_t* t_full = bars + 2 * p.slots;   // [2] MMA commit -> epilogue group
  uint64_t* t_empty = t_full + 2;          // [2] epilogue group (4 warps) -> MMA
  uint64_t* st_full = t_full + 4;          // [nstage] every loader lane's copies landed
  uint64_t* st_empty = st_full + p.nstage; // [nstage] the producer warps are done with it
  uint64_t* kn_full = st_empty + p.nstage; // [kKnRing] key norms of step n written (64)
  uint64_t* kn_empty = kn_full + kKnRing;  // [kKnRing] read by the epilogue group (4 warps)
  float* s_kn = reinterpret_cast<float*>(misc + 256 + 1024 + 4 * 32 * 4 + 256 + 16);  // [kKnRing][128]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = blockIdx.x % p.n_grp;
  const int b0 = grp * p.gsize;
  const int nbl = min(p.gsize, p.nb - b0);
  constexpr int kt = TcShape<BD>::kKt;
  const uint32_t a_slot_bytes = kTcRows * kt * 2;
  const uint32_t b_blk_bytes = (uint32_t)p.k * kt * 2;
  const int dt = p.key_dtype;

  // ---- setup: tables, barriers, TMEM, resident B operands -------------------
  for (int i = tid; i < p.d; i += kTcThreads) s_pcol[i] = (int16_t)((p.perm ? p.perm[i] : i) * p.es);
  for (int i = tid; i < 32; i += kTcThreads) s_cmax[i] = 0.f;
  if (tid == 0) {
    int h = 0;
    for (int b = 0; b < p.nb; ++b) {
      const uint8_t hv = p.heavy ? p.heavy[b] : 0;
      s_heavy[b] = hv;
      s_hpos[b] = (uint8_t)h;
      h += hv ? 1 : 0;
    }
    for (int s = 0; s < p.slots; ++s) {
      mbar_init(a_full + s, kTcProdThreads);
      mbar_init(a_empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(t_full + s, 1);
      mbar_init(t_empty + s, 4);
    }
    for (int s = 0; s < p.nstage; ++s) {
      mbar_init(st_full + s, 32);
      mbar_init(st_empty + s, kTcProdThreads / 32);
    }
    for (int s = 0; s < kKnRing; ++s) {
      mbar_init(kn_full + s, kTcProdThreads);
      mbar_init(kn_empty + s, 4);
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  // per-block scale: 2^(1 - e) with max |c| = m * 2^e, m in [0.5, 1)
  for (int bl = warp; bl < nbl; bl += kTcThreads / 32) {
    const float* cb = p.cents + (size_t)(b0 + bl) * p.k * BD;
    float m = 0.f;
    for (int i = lane; i < p.k * BD; i += 32) m = fmaxf(m, fabsf(cb[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) {
      int e = 0;
      float sc = 1.f;
      if (m > 0.f && m <= 3.0e38f) {
        frexpf(m, &e);
        sc = ldexpf(1.f, 1 - e);
      }
      s_scale[bl] = sc;
      // The gap test bounds relative errors; outside [2^-100, 2^100] (unscaled)
      // the reference's distances can underflow or overflow, so such rows
      // always take the exact path.
      s_slo[bl] = ldexpf(1.f, -100 + 2 * (1 - e));
      s_shi[bl] = ldexpf(1.f, 100 + 2 * (1 - e));
    }
  }
  if (warp == kTcMmaWarp) {
    tc_alloc(s_tmem, 512);
    tc_relinquish();
  }
  __syncthreads();
  for (int i = tid; i < nbl * p.k * BD / 4; i += kTcThreads) {
    reinterpret_cast<float4*>(s_cf)[i] =
        reinterpret_cast<const float4*>(p.cents + (size_t)b0 * p.k * BD)[i];
  }
  // B rows: [ch | cl | ch | csq_h, csq_l, 0...] per centroid, scaled
  for (int row = tid; row < nbl * p.k; row += kTcThreads) {
    const int bl = row / p.k, c = row - bl * p.k;
    const float sc = s_scale[bl];
    const float* src = p.cents + ((size_t)(b0 + bl) * p.k + c) * BD;
    uint8_t* dst = s_b + (size_t)bl * b_blk_bytes;
    __half hv[kt];
#pragma unroll
    for (int j = 0; j < kt; ++j) hv[j] = __ushort_as_half(0);
    float csq = 0.f;
#pragma unroll
    for (int j = 0; j < BD; ++j) {
      const float x = src[j] * sc;
      csq = fmaf(x, x, csq);
      const __half h = __float2half_rn(x);
      const __half l = __float2half_rn(x - __half2float(h));
      hv[j] = h;
      hv[BD + j] = l;
      hv[2 * BD + j] = h;
    }
    const __half ch = __float2half_rn(csq);
    hv[3 * BD] = ch;
    hv[3 * BD + 1] = __float2half_rn(csq - __half2float(ch));
#pragma unroll
    for (int e = 0; e < kt; e += 2) {
      *reinterpret_cast<__half2*>(dst + kmaj_off(c, e, kt)) = __halves2half2(hv[e], hv[e + 1]);
    }
    atomicMax(reinterpret_cast<int*>(s_cmax) + bl, __float_as_int(csq));  // csq >= 0
  }
  // A slots: elements [2*BD, 3*BD) = 0 (stays 0 for fp16 keys), [3*BD, kt) = 1, 1, 0, ...
  for (int i = tid; i < p.slots * kTcRows; i += kTcThreads) {
    const int s = i / kTcRows, r = i - s * kTcRows;
    uint8_t* dst = s_a + (size_t)s * a_slot_bytes;
    for (int e = 2 * BD; e < kt; e += 2) {
      const float v = e == 3 * BD ? 1.f : 0.f;
      *reinterpret_cast<__half2*>(dst + kmaj_off(r, e, kt)) =
          __halves2half2(__float2half_rn(v), __float2half_rn(v));
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  const int64_t tstride = gridDim.x / p.n_grp;
  const int64_t tfirst = blockIdx.x / p.n_grp;

  if (warp >= kTcProdWarp0 && warp < kTcLoadWarp) {
    // ---------------------------------------------------------- producers
    const int pt = tid - kTcProdWarp0 * 32;  // rows pt, pt + 64 of the tile
    uint32_t n = 0, li = 0;
    bool ok = true;
    // After an abandoned wait the loops keep running without work.
    for (int64_t tile = tfirst; tile < p.n_tiles; tile += tstride, ++li) {
      const int sb = li % p.nstage;
      if (ok) ok = tc_wait(st_full + sb, (li / p.nstage) & 1, s_abort, p);
      const uint8_t* st = s_stage + (size_t)sb * p.stage_bytes;
      for (int bl = 0; bl < nbl; ++bl, ++n) {
        const int b = b0 + bl;
        const uint32_t slot = n % p.slots;
        if (ok) ok = tc_wait(a_empty + slot, ((n / p.slots) & 1) ^ 1, s_abort, p);
        if (ok) ok = tc_wait(kn_empty + n % kKnRing, ((n / kKnRing) & 1) ^ 1, s_abort, p);
        if (!ok) continue;
        uint8_t* dst = s_a + (size_t)slot * a_slot_bytes;
        float* kn_out = s_kn + (n % kKnRing) * kTcRows;
        const bool heavy = s_heavy[b] != 0;
        const float sc = s_scale[bl];
        for (int row = pt; row < kTcRows; row += kTcProdThreads) {
          float x[BD];
#pragma unroll
          for (int j = 0; j < BD; ++j) x[j] = stage_val(st, p.stage_stride, row, s_pcol[b * BD + j], dt);
          if (heavy) {
            const int64_t g = tile / p.tpg;
            const int64_t t = (tile - g * p.tpg) * kTcRows + row;
            if (t < p.rpg) {
              if (p.out_heavy) {
                uint16_t* hd = p.out_heavy + g * p.hgs + t * p.hrs + s_hpos[b] * BD;
#pragma unroll
                for (int j = 0; j < BD; ++j) hd[j] = f2h(x[j]);
              }
              if (p.out_pt) {
                float* pd = p.out_pt + (g * p.rpg + t) * (int64_t)p.nb * BD + b * BD;
#pragma unroll
                for (int j = 0; j < BD; ++j) pd[j] = x[j];
              }
            }
            continue;
          }
          // -2 * (x * sc) as fp16 hi (and lo unless the keys are fp16, whose
          // power-of-two scaling is exact); the scaled squared key norm, NaN
          // when a scaled value does not fit fp16 (forces the exact path)
          uint32_t hw[BD / 2], lw[BD / 2];
          float kn = 0.f;
          bool fits = true;
#pragma unroll
          for (int j = 0; j < BD; j += 2) {
            const float x0 = x[j] * sc, x1 = x[j + 1] * sc;
            kn = fmaf(x1, x1, fmaf(x0, x0, kn));
            fits = fits && fabsf(x0) <= 32752.f && fabsf(x1) <= 32752.f;  // false for NaN / inf
            const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
            hw[j / 2] = pack_h2(-2.f * __half2float(h0), -2.f * __half2float(h1));
            if (dt != SS_F16) {
              lw[j / 2] = pack_h2(-2.f * (x0 - __half2float(h0)), -2.f * (x1 - __half2float(h1)));
            }
          }
          if constexpr (BD % 8 == 0) {
#pragma unroll
            for (int q = 0; q < BD; q += 8) {
              const uint4 hv = make_uint4(hw[q / 2], hw[q / 2 + 1], hw[q / 2 + 2], hw[q / 2 + 3]);
              *reinterpret_cast<uint4*>(dst + kmaj_off(row, q, kt)) = hv;
              *reinterpret_cast<uint4*>(dst + kmaj_off(row, BD + q, kt)) = hv;
              if (dt != SS_F16) {
                *reinterpret_cast<uint4*>(dst + kmaj_off(row, 2 * BD + q, kt)) =
                    make_uint4(lw[q / 2], lw[q / 2 + 1], lw[q / 2 + 2], lw[q / 2 + 3]);
              }
            }
          } else {
#pragma unroll
            for (int q = 0; q < BD; q += 2) {
              *reinterpret_cast<uint32_t*>(dst + kmaj_off(row, q, kt)) = hw[q / 2];
              *reinterpret_cast<uint32_t*>(dst + kmaj_off(row, BD + q, kt)) = hw[q / 2];
              if (dt != SS_F16) *reinterpret_cast<uint32_t*>(dst + kmaj_off(row, 2 * BD + q, kt)) = lw[q / 2];
            }
          }
          kn_out[row] = fits ? kn : __int_as_float(0x7fc00000);
        }
        fence_proxy_async_smem();
        mbar_arrive(a_full + slot);
        mbar_arrive(kn_full + n % kKnRing);
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(st_empty + sb);
    }
  } else if (warp == kTcLoadWarp) {
    // ---------------------------------------------------------- tile loader
    // Stages key tiles as far ahead as the stage ring allows: 16-byte cp.async
    // copies per lane (rows past the group's end read nothing and stage
    // zeros), then one arrival per lane once its copies have landed.
    const uint32_t vr = (uint32_t)p.d * p.es / 16;  // 16-byte chunks per key row
    uint32_t li = 0;
    for (int64_t tile = tfirst; tile < p.n_tiles; tile += tstride, ++li) {
      const int buf = li % p.nstage;
      const uint32_t use = li / p.nstage;
      if (use > 0 && !__all_sync(0xffffffffu, tc_wait(st_empty + buf, (use - 1) & 1, s_abort, p))) break;
      if (tile == p.skip_tile) continue;  // test hook: this stage never fills
      const int64_t g = tile / p.tpg;
      const int64_t t0 = (tile - g * p.tpg) * kTcRows;
      const uint8_t* src0 =
          reinterpret_cast<const uint8_t*>(p.keys) + (g * p.kgs + t0 * p.krs) * p.es;
      const uint32_t dst0 = smem_u32(s_stage + (size_t)buf * p.stage_bytes);
      for (uint32_t v = lane; v < kTcRows * vr; v += 32) {
        const uint32_t rr = v / vr, cv = v - rr * vr;
        const bool in = t0 + rr < p.rpg;
        cp_async16(dst0 + rr * p.stage_stride + cv * 16,
                   in ? src0 + (int64_t)rr * p.krs * p.es + cv * 16 : src0, in ? 16u : 0u);
      }
      cp_async_mbar_arrive(st_full + buf);
    }
    // copies of this lane still in flight after a give-up land before exit
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == kTcMmaWarp) {
    // TMEM owner: allocated above, released below; the epilogue groups
    // issue their own MMAs.
  } else {
    // ---------------------------------------------------------- epilogue
    const int eg = warp >> 2;          // 0: even steps, 1: odd steps
    const int sub = warp & 3;          // TMEM lane quarter
    const int row = sub * 32 + lane;   // tile row of this thread
    const uint32_t tbase = tmem + ((uint32_t)(sub * 32) << 16) + eg * 256;
    const int nch = p.k / 32;
    const int64_t ntl = tfirst < p.n_tiles ? (p.n_tiles - tfirst + tstride - 1) / tstride : 0;
    const uint32_t nsteps = (uint32_t)(ntl * nbl);
    // Lane 0 of the group's first warp issues the group's MMAs (steps
    // eg, eg + 2, ...) into the group's TMEM buffer, so neither group waits
    // for the other.
    const bool issuer = sub == 0 && lane == 0;
    const uint32_t idesc = instr_desc_f16(p.k);
    const uint32_t a0 = smem_u32(s_a), bb0 = smem_u32(s_b);
    auto issue_mma = [&](uint32_t q) -> bool {
      const uint32_t slot = q % p.slots;
      const int qbl = (int)(q % nbl);
      if (!tc_wait(t_empty + eg, ((q >> 1) & 1) ^ 1, s_abort, p)) return false;
      if (!tc_wait(a_full + slot, (q / p.slots) & 1, s_abort, p)) return false;
      tc_fence_after();
      const uint32_t a_addr = a0 + slot * a_slot_bytes;
      const uint32_t b_addr = bb0 + qbl * b_blk_bytes;
#pragma unroll
      for (int j = 0; j < kt / 16; ++j) {
        tc_mma_f16(tmem + eg * 256, smem_desc(a_addr + j * 256, 128, kt * 16),
                   smem_desc(b_addr + j * 256, 128, kt * 16), idesc, j > 0 ? 1u : 0u);
      }
      tc_commit(a_empty + slot);
      tc_commit(t_full + eg);
      return true;
    };
    bool ok = true;
    int64_t last = -1;  // last step this group's issuer launched
    if (sub == 0) {
      bool r = true;
      if (issuer && (uint32_t)eg < nsteps) { r = issue_mma(eg); last = eg; }
      ok = __shfl_sync(0xffffffffu, r, 0);
    }
    for (uint32_t n = eg; n < nsteps && ok; n += 2) {
      const uint32_t li = n / nbl;
      const int bl = (int)(n - li * nbl);
      const int64_t tile = tfirst + (int64_t)li * tstride;
      const int64_t g = tile / p.tpg;
      const int64_t t = (tile - g * p.tpg) * kTcRows + row;
      const bool valid = t < p.rpg;
      {
        const int b = b0 + bl;
        ok = __all_sync(0xffffffffu, tc_wait(t_full + eg, (n >> 1) & 1, s_abort, p));
        if (!ok) break;
        tc_fence_after();
        const bool heavy = s_heavy[b] != 0;
        int idx = 0;
        bool need = false;
        // the producers' scaled squared key norm of this row (NaN: exact path)
        ok = __all_sync(0xffffffffu, tc_wait(kn_full + n % kKnRing, (n / kKnRing) & 1, s_abort, p));
        if (!ok) break;
        const float kn = s_kn[(n % kKnRing) * kTcRows + row];
        __syncwarp();
        if (lane == 0) mbar_arrive(kn_empty + n % kKnRing);
        if (!heavy) {
          // One pass over the row's V (ALU pipe): the minima of two partitions
          // of the columns, ma[c >> 4] (16 runs of 16 columns) and mb[c & 15]
          // (16 residue classes), one three-input min per two columns each.
          // Two distinct columns differ in their high or low nibble, so some
          // other column lies within T of the minimum s1 exactly when, in one
          // of the partitions, a second group's minimum is below s1 + T. If
          // each partition has a single group below it, the winner is the
          // column (that ma group, that mb group).
          const float inf = __int_as_float(0x7f800000);
          float ma[16], mb[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) { ma[q] = inf; mb[q] = inf; }
#pragma unroll
          for (int ch = 0; ch < 8; ch += 2) {
            if (ch < nch) {
              uint32_t v0[32], v1[32];
              tc_ld32(tbase + ch * 32, v0);
              tc_ld32(tbase + (ch + 1) * 32, v1);  // nch is even
              tc_wait_ld();
              float a0 = inf, a1 = inf, a2 = inf, a3 = inf;
#pragma unroll
              for (int j = 0; j < 16; j += 2) {
                a0 = fmin3(a0, __uint_as_float(v0[j]), __uint_as_float(v0[j + 1]));
                a1 = fmin3(a1, __uint_as_float(v0[j + 16]), __uint_as_float(v0[j + 17]));
                a2 = fmin3(a2, __uint_as_float(v1[j]), __uint_as_float(v1[j + 1]));
                a3 = fmin3(a3, __uint_as_float(v1[j + 16]), __uint_as_float(v1[j + 17]));
              }
              ma[2 * ch] = a0;
              ma[2 * ch + 1] = a1;
              ma[2 * ch + 2] = a2;
              ma[2 * ch + 3] = a3;
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                mb[j] = fmin3(mb[j], __uint_as_float(v0[j]), __uint_as_float(v0[j + 16]));
                mb[j] = fmin3(mb[j], __uint_as_float(v1[j]), __uint_as_float(v1[j + 16]));
              }
            }
          }
          float s1 = inf;
#pragma unroll
          for (int q = 0; q < 16; q += 2) s1 = fmin3(s1, ma[q], ma[q + 1]);
          const float sn = kn + s_cmax[bl];
          const float thr = s1 + sn * kTieRel;
          int na = 0, nbm = 0, wa = 0, wb = 0;
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            if (ma[q] < thr) { ++na; wa = q; }
            if (mb[q] < thr) { ++nbm; wb = q; }
          }
          need = valid && !(na == 1 && nbm == 1 && sn >= s_slo[bl] && sn <= s_shi[bl]);
          idx = min(wa * 16 + wb, p.k - 1);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(t_empty + eg);
        if (sub == 0) {
          bool r = true;
          if (issuer && n + 2 < nsteps) { r = issue_mma(n + 2); last = n + 2; }
          ok = __shfl_sync(0xffffffffu, r, 0);
          if (!ok) break;
        }
        uint32_t m = __ballot_sync(0xffffffffu, need);
        // rows to re-score load their permuted block values (global memory,
        // usually L2) all at once, then the warp scores them one by one
        float kown[BD];
        if (need) {
          const int64_t base = g * p.kgs + t * p.krs;
#pragma unroll
          for (int j = 0; j < BD; ++j) kown[j] = load_as_f32(p.keys, dt, base + s_pcol[b * BD + j] / p.es);
        }
        while (m) {
          const int src = __ffs(m) - 1;
          m &= m - 1;
          float kk[BD];
#pragma unroll
          for (int j = 0; j < BD; ++j) kk[j] = __shfl_sync(0xffffffffu, kown[j], src);
          const int bi = exact_rescan<BD>(kk, s_cf + (size_t)bl * p.k * BD, p.k, p.dist_mode, lane);
          if (lane == src) idx = bi;
        }
        if (valid) p.out_idx[g * p.igs + t * p.irs + b] = (uint8_t)idx;
      }
    }
    // After an abandoned wait, let this group's launched MMAs finish before
    // the TMEM is released (bounded).
    if (!ok && issuer && last >= 0) mbar_wait_bounded(t_full + eg, (uint32_t)(last >> 1) & 1, 1000000ull);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kTcMmaWarp) {
    tc_fence_after();
    tc_dealloc(tmem, 512);
  }
}

}  // namespace

// ---------------------------------------------------------------- host side
std::atomic<int64_t> g_tc_wait_ns{0};     // ss_set_assign_wait (tests)
std::atomic<int64_t> g_tc_skip_tile{0};

// Returns SS_ERR_UNSUPPORTED when the tensor-core path does not apply.
int launch_vq_assign_tc(const void* keys, int key_dtype, int64_t n_groups, int64_t rpg,
                        int64_t kgs, int64_t krs, int d, const int32_t* perm,
                        const float* cents, int bd, int k, const uint8_t* heavy,
                        uint8_t* out_idx, int64_t igs, int64_t irs, uint16_t* out_heavy,
                        int64_t hgs, int64_t hrs, float* out_pt, int dist_mode,
                        cudaStream_t st) {
  const int es = key_dtype == SS_F32 ? 4 : 2;
  if (!(bd == 4 || bd == 8 || bd == 16)) return SS_ERR_UNSUPPORTED;
  if (k % 64 != 0 || k < 64 || k > 256) return SS_ERR_UNSUPPORTED;
  if ((d * es) % 16 != 0 || d * es > 512) return SS_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(keys) & 15) != 0) return SS_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(cents) & 15) != 0) return SS_ERR_UNSUPPORTED;
  if (((kgs * es) & 15) != 0 || ((krs * es) & 15) != 0 || krs < d) return SS_ERR_UNSUPPORTED;
  const int nb = d / bd;
  const int kt = bd == 4 ? TcShape<4>::kKt : bd == 8 ? TcShape<8>::kKt : TcShape<16>::kKt;
  const uint32_t stage_stride = (uint32_t)(d * es + 16);
  const uint32_t stage_bytes = kTcRows * stage_stride;
  const uint32_t misc_bytes = 256 + 1024 + 4 * 32 * 4 + 256 + 16 + kKnRing * kTcRows * 4;
  // per block: the B operand plus a float32 copy of the centroids (exact re-scans)
  const uint32_t b_blk = (uint32_t)k * kt * 2, cf_blk = (uint32_t)k * bd * 4;
  const uint32_t a_slot = kTcRows * kt * 2;
  const uint32_t limit = 227 * 1024;
  // Prefer 3 staged tiles and 3 A slots; shrink both for wide blocks / fp32 keys.
  int nstage = 0, slots = 0, gsize = 0;
  const int cand[4][2] = {{3, 3}, {2, 3}, {2, 2}, {1, 2}};
  for (const auto& c : cand) {
    const uint32_t fixed = c[1] * a_slot + c[0] * stage_bytes + misc_bytes;
    const int gs = fixed < limit ? (int)((limit - fixed) / (b_blk + cf_blk)) : 0;
    if (gs >= 2 || (gs >= 1 && c[0] == 1) || (gs >= nb)) {
      nstage = c[0]; slots = c[1]; gsize = gs;
      break;
    }
    if (gs >= 1 && gsize == 0) { nstage = c[0]; slots = c[1]; gsize = gs; }
  }
  if (gsize < 1) return SS_ERR_UNSUPPORTED;
  if (gsize > nb) gsize = nb;
  if (gsize > 32) gsize = 32;
  const int n_grp = (nb + gsize - 1) / gsize;
  gsize = (nb + n_grp - 1) / n_grp;  // balance the groups
  TcParams p{};
  p.keys = keys; p.key_dtype = key_dtype; p.es = es;
  p.n_groups = n_groups; p.rpg = rpg; p.kgs = kgs; p.krs = krs;
  p.d = d; p.nb = nb; p.k = k; p.bd = bd; p.kt = kt;
  p.perm = perm; p.cents = cents; p.heavy = heavy; p.out_idx = out_idx;
  p.igs = igs; p.irs = irs; p.out_heavy = out_heavy; p.hgs = hgs; p.hrs = hrs;
  p.out_pt = out_pt; p.dist_mode = dist_mode;
  p.n_grp = n_grp; p.gsize = gsize; p.slots = slots; p.nstage = nstage;
  p.tpg = (rpg + kTcRows - 1) / kTcRows;
  p.wait_ns = g_tc_wait_ns > 0 ? static_cast<uint64_t>(g_tc_wait_ns) : kTcWaitNs;
  p.skip_tile = g_tc_skip_tile > 0 ? g_tc_skip_tile - 1 : -1;
  p.sink = error_sink();
  p.n_tiles = n_groups * p.tpg;
  uint32_t off = 0;
  p.off_stage = off; off += nstage * stage_bytes;   // 1024-aligned sizes first
  p.off_b = off; off += (uint32_t)gsize * b_blk;
  p.off_a = off; off += slots * a_slot;
  p.off_cf = off; off += (uint32_t)gsize * cf_blk;
  p.off_misc = off; off += misc_bytes;
  p.stage_bytes = stage_bytes;
  p.stage_stride = stage_stride;
  if (off > limit) return SS_ERR_UNSUPPORTED;
  // More than half an SM's shared memory: exactly one CTA (and one 512-column
  // TMEM allocation) per SM, so allocations never wait on each other.
  uint32_t smem = off;
  if (smem < 120 * 1024) smem = 120 * 1024;
  int per_grp = sm_count() / n_grp;
  if (per_grp < 1) per_grp = 1;
  if (per_grp > p.n_tiles) per_grp = (int)p.n_tiles;
  const int grid = per_grp * n_grp;
#define SS_LAUNCH_TC(BDV)                                                                   \
  case BDV:                                                                                 \
    cudaFuncSetAttribute(vq_assign_tc_kernel<BDV>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                         (int)smem);                                                        \
    vq_assign_tc_kernel<BDV><<<grid, kTcThreads, smem, st>>>(p);                       \
    break;
  switch (bd) {
    SS_LAUNCH_TC(4)
    SS_LAUNCH_TC(8)
    SS_LAUNCH_TC(16)
  }
#undef SS_LAUNCH_TC
  return check_launch("ss_vq_assign (tensor cores)");
}

}  // namespace ss

using namespace ss;

extern "C" int ss_set_assign_wait(int64_t wait_limit_ns, int64_t skip_tile) {
  g_tc_wait_ns.store(wait_limit_ns);
  g_tc_skip_tile.store(skip_tile);
  return SS_OK;
}

extern "C" int ss_vq_assign_check(void* stream) {
  cudaError_t e = cudaStreamSynchronize(as_stream(stream));
  unsigned int v = 0;
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_assign_status, sizeof(v));
  if (e == cudaSuccess && v) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_assign_status, &z, sizeof(z));
  }
  if (e != cudaSuccess) {
    return fail(SS_ERR_CUDA, std::string("ss_vq_assign_check: ") + cudaGetErrorString(e));
  }
  if (v) return fail(SS_ERR_TIMEOUT, "ss_vq_assign: a tensor-core pipeline wait timed out");
  return SS_OK;
}
