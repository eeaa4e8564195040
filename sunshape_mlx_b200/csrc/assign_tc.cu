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
// The epilogue (one thread per row) keeps the smallest and second smallest V
// with the centroid index packed into the low mantissa bits. Error analysis
// (u = 2^-24, S = ||k||^2 + max_c ||c||^2, all in scaled units):
//   |reference distance - exact real distance| <= 64u * S (both modes),
//   |V - (exact distance - ||k||^2)|         <= 2^-16 * S (fp16 splits, the
//        dropped kl*cl term, fp32 accumulation of <= 64 exact products),
//   |packed V - V|                            <= 2^-14 * S (8 low bits).
// So when second - first > 2^-12 * S no other centroid can have a reference
// distance <= the winner's, and the winner is the reference's argmin. Rows
// where that gap test fails (or whose values are not finite, or whose scaled
// key does not fit fp16) are re-scored exactly by the whole warp in the
// reference order, ties to the lowest index (np.argmin, kernels.py:1020).
//
// CTA roles (416 threads, one CTA per SM, persistent over row tiles):
//   warps 0-7   epilogue: warp w reads TMEM lanes 32*(w%4)..+31; warps 0-3
//               take even sequence steps (TMEM buffer 0), warps 4-7 odd ones
//   warp 8      TMEM allocation; lane 0 issues the MMAs
//   warps 9-12  producers: stage 128 key rows (coalesced 16-byte loads into a
//               padded shared-memory tile), gather the permuted block, build
//               the A operand in the canonical no-swizzle K-major layout
// A sequence step is one (tile, block) pair; blocks of a CTA are a contiguous
// group of the codec's blocks whose B operands stay resident in shared memory.
#include "common.cuh"
#include "vq_math.cuh"

namespace ss {

__device__ unsigned int g_assign_status = 0;  // sticky: 1 = a pipeline wait gave up

namespace {

constexpr int kTcRows = 128;            // MMA M (rows per tile)
constexpr int kTcMmaWarp = 8;
constexpr int kTcProdWarp0 = 9;
constexpr int kTcProdThreads = 128;
constexpr int kTcThreads = (kTcProdWarp0 * 32) + kTcProdThreads;  // 416
constexpr uint64_t kTcWaitNs = 2000000000ull;                      // 2 s per wait
constexpr float kTieRel = 1.0f / 4096.0f;                           // 2^-12

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
  int64_t n_rows, n_tiles;
  // dynamic shared-memory offsets (bytes)
  uint32_t off_b, off_a, off_kn, off_stage, off_misc;
  uint32_t stage_stride;  // bytes per staged row (d*es + 4)
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

__device__ __forceinline__ uint32_t pack_halves(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
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

struct Bar {
  uint64_t* a_full;   // [slots] producers -> MMA (128 arrivals)
  uint64_t* a_empty;  // [slots] epilogue group -> producers (4 arrivals)
  uint64_t* t_full;   // [2] MMA commit -> epilogue group
  uint64_t* t_empty;  // [2] epilogue group -> MMA (4 arrivals)
};

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (global_ns() - t0 > kTcWaitNs) {
      *abort = 1;
      atomicOr(&g_assign_status, 1u);
      return false;
    }
  }
}

__device__ __forceinline__ void key_row_addr(const TcParams& p, int64_t r, int64_t& g,
                                             int64_t& t) {
  g = r / p.rpg;
  t = r - g * p.rpg;
}

// Exact re-score of one (row, block) by the whole warp, reference order,
// sequential '<' semantics of the reference loop: the first index whose
// distance is below every earlier one; a NaN distance at index 0 keeps 0.
template <int BD>
__device__ int exact_rescan(const TcParams& p, const int16_t* s_perm, int64_t r, int b,
                            int lane) {
  int64_t g, t;
  key_row_addr(p, r, g, t);
  const int64_t base = g * p.kgs + t * p.krs;
  float kk[BD];
#pragma unroll
  for (int j = 0; j < BD; ++j) kk[j] = load_as_f32(p.keys, p.key_dtype, base + s_perm[b * BD + j]);
  const float* cb = p.cents + (size_t)b * p.k * BD;
  float best = __int_as_float(0x7f800000);
  int bi = 0x7fffffff;
  float d0 = 0.f;
  for (int c = lane; c < p.k; c += 32) {
    float cc[BD];
#pragma unroll
    for (int j = 0; j < BD; ++j) cc[j] = __ldg(cb + (size_t)c * BD + j);
    const float dd = p.dist_mode == 0 ? dist_direct<BD>(kk, cc) : dist_expanded<BD>(kk, cc);
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

template <int BD>
__global__ void __launch_bounds__(kTcThreads, 1) vq_assign_tc_kernel(TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* s_b = smem + p.off_b;
  uint8_t* s_a = smem + p.off_a;
  float* s_kn = reinterpret_cast<float*>(smem + p.off_kn);
  uint8_t* s_stage = smem + p.off_stage;
  uint8_t* misc = smem + p.off_misc;
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc);              // 2*slots + 4
  int16_t* s_perm = reinterpret_cast<int16_t*>(misc + 8 * 40);     // [d]
  float* s_scale = reinterpret_cast<float*>(misc + 8 * 40 + 2048); // [gsize]
  float* s_cmax = s_scale + 32;                                     // [gsize]
  float* s_slo = s_cmax + 32;   // [gsize] scaled S below which fp32 distances may underflow
  float* s_shi = s_slo + 32;    // [gsize] scaled S above which they may overflow
  uint8_t* s_heavy = reinterpret_cast<uint8_t*>(s_shi + 32);        // [nb]
  uint8_t* s_hpos = s_heavy + 128;                                  // [nb]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(s_hpos + 128);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  Bar bar{bars, bars + p.slots, bars + 2 * p.slots, bars + 2 * p.slots + 2};
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = blockIdx.x % p.n_grp;
  const int b0 = grp * p.gsize;
  const int nbl = min(p.gsize, p.nb - b0);
  constexpr int kt = TcShape<BD>::kKt;
  const uint32_t a_slot_bytes = kTcRows * kt * 2;
  const uint32_t b_blk_bytes = (uint32_t)p.k * kt * 2;

  // ---- setup: tables, barriers, TMEM, resident B operands -------------------
  for (int i = tid; i < p.d; i += kTcThreads) s_perm[i] = (int16_t)(p.perm ? p.perm[i] : i);
  if (tid == 0) {
    int h = 0;
    for (int b = 0; b < p.nb; ++b) {
      const uint8_t hv = p.heavy ? p.heavy[b] : 0;
      s_heavy[b] = hv;
      s_hpos[b] = (uint8_t)h;
      h += hv ? 1 : 0;
    }
    for (int s = 0; s < p.slots; ++s) {
      mbar_init(bar.a_full + s, kTcProdThreads);
      mbar_init(bar.a_empty + s, 4);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar.t_full + s, 1);
      mbar_init(bar.t_empty + s, 4);
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  for (int i = tid; i < 32; i += kTcThreads) s_cmax[i] = 0.f;
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
      __half2 pr = __halves2half2(hv[e], hv[e + 1]);
      *reinterpret_cast<__half2*>(dst + kmaj_off(c, e, kt)) = pr;
    }
    atomicMax(reinterpret_cast<int*>(s_cmax) + bl, __float_as_int(csq));  // csq >= 0
  }
  // constant part of every A slot: elements [3*BD, kt) = 1, 1, 0, ...
  for (int i = tid; i < p.slots * kTcRows; i += kTcThreads) {
    const int s = i / kTcRows, r = i - s * kTcRows;
    uint8_t* dst = s_a + (size_t)s * a_slot_bytes;
    for (int e = 3 * BD; e < kt; e += 2) {
      const __half lo = __float2half_rn(e == 3 * BD ? 1.f : 0.f);
      const __half hi = __float2half_rn(e == 3 * BD ? 1.f : 0.f);
      *reinterpret_cast<__half2*>(dst + kmaj_off(r, e, kt)) = __halves2half2(lo, hi);
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  const int64_t tstride = gridDim.x / p.n_grp;
  const int64_t t0 = blockIdx.x / p.n_grp;

  if (warp >= kTcProdWarp0) {
    // ---------------------------------------------------------- producers
    const int pt = tid - kTcProdWarp0 * 32;  // 0..127 = tile row
    const uint32_t rb = (uint32_t)p.d * p.es, vr = rb / 16;
    uint32_t n = 0;
    bool ok = true;
    // After an abandoned wait the loops keep running without work so that
    // every producer thread still reaches the same named barriers.
    for (int64_t tile = t0; tile < p.n_tiles; tile += tstride) {
      named_bar_sync(1, kTcProdThreads);  // previous tile's gathers are done
      for (uint32_t v = pt; v < kTcRows * vr; v += kTcProdThreads) {
        const uint32_t rr = v / vr, cv = v - rr * vr;
        const int64_t r = tile * kTcRows + rr;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (r < p.n_rows) {
          int64_t g, t;
          key_row_addr(p, r, g, t);
          const uint8_t* src = reinterpret_cast<const uint8_t*>(p.keys) +
                               (g * p.kgs + t * p.krs) * p.es + cv * 16;
          val = __ldg(reinterpret_cast<const uint4*>(src));
        }
        uint32_t* dst = reinterpret_cast<uint32_t*>(s_stage + rr * p.stage_stride + cv * 16);
        dst[0] = val.x; dst[1] = val.y; dst[2] = val.z; dst[3] = val.w;
      }
      named_bar_sync(1, kTcProdThreads);
      const int64_t r = tile * kTcRows + pt;
      const bool valid = r < p.n_rows;
      const uint8_t* srow = s_stage + pt * p.stage_stride;
      for (int bl = 0; bl < nbl; ++bl, ++n) {
        const int b = b0 + bl;
        const uint32_t slot = n % p.slots;
        if (ok) ok = tc_wait(bar.a_empty + slot, ((n / p.slots) & 1) ^ 1, s_abort);
        if (!ok) continue;
        float x[BD];
#pragma unroll
        for (int j = 0; j < BD; ++j) {
          const int dd = s_perm[b * BD + j];
          if (p.es == 4) {
            x[j] = *reinterpret_cast<const float*>(srow + dd * 4);
          } else {
            const uint16_t u = *reinterpret_cast<const uint16_t*>(srow + dd * 2);
            x[j] = p.key_dtype == SS_F16 ? h2f(u) : bf2f(u);
          }
        }
        if (s_heavy[b]) {
          if (valid) {
            int64_t g, t;
            key_row_addr(p, r, g, t);
            if (p.out_heavy) {
              uint16_t* dst = p.out_heavy + g * p.hgs + t * p.hrs + s_hpos[b] * BD;
#pragma unroll
              for (int j = 0; j < BD; ++j) dst[j] = f2h(x[j]);
            }
            if (p.out_pt) {
              float* dst = p.out_pt + r * (int64_t)p.nb * BD + b * BD;
#pragma unroll
              for (int j = 0; j < BD; ++j) dst[j] = x[j];
            }
          }
        } else {
          const float sc = s_scale[bl];
          float kn = 0.f;
          bool fits = true;
          __half ah[BD], al[BD];
#pragma unroll
          for (int j = 0; j < BD; ++j) {
            const float xs = x[j] * sc;
            kn = fmaf(xs, xs, kn);
            fits = fits && (fabsf(xs) <= 32752.f);  // false for NaN / inf too
            const __half h = __float2half_rn(xs);
            const __half l = __float2half_rn(xs - __half2float(h));
            ah[j] = __float2half_rn(-2.f * __half2float(h));
            al[j] = __float2half_rn(-2.f * __half2float(l));
          }
          uint8_t* dst = s_a + (size_t)slot * a_slot_bytes;
          if constexpr (BD % 8 == 0) {
#pragma unroll
            for (int q = 0; q < BD; q += 8) {
              uint4 hv, lv;
              hv.x = pack_halves(ah[q], ah[q + 1]); hv.y = pack_halves(ah[q + 2], ah[q + 3]);
              hv.z = pack_halves(ah[q + 4], ah[q + 5]); hv.w = pack_halves(ah[q + 6], ah[q + 7]);
              lv.x = pack_halves(al[q], al[q + 1]); lv.y = pack_halves(al[q + 2], al[q + 3]);
              lv.z = pack_halves(al[q + 4], al[q + 5]); lv.w = pack_halves(al[q + 6], al[q + 7]);
              *reinterpret_cast<uint4*>(dst + kmaj_off(pt, q, kt)) = hv;
              *reinterpret_cast<uint4*>(dst + kmaj_off(pt, BD + q, kt)) = hv;
              *reinterpret_cast<uint4*>(dst + kmaj_off(pt, 2 * BD + q, kt)) = lv;
            }
          } else {
#pragma unroll
            for (int q = 0; q < BD; q += 2) {
              const uint32_t hv = pack_halves(ah[q], ah[q + 1]);
              const uint32_t lv = pack_halves(al[q], al[q + 1]);
              *reinterpret_cast<uint32_t*>(dst + kmaj_off(pt, q, kt)) = hv;
              *reinterpret_cast<uint32_t*>(dst + kmaj_off(pt, BD + q, kt)) = hv;
              *reinterpret_cast<uint32_t*>(dst + kmaj_off(pt, 2 * BD + q, kt)) = lv;
            }
          }
          s_kn[slot * kTcRows + pt] = fits ? kn : __int_as_float(0x7fc00000);
          fence_proxy_async_smem();
        }
        mbar_arrive(bar.a_full + slot);
      }
    }
  } else if (warp == kTcMmaWarp) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = instr_desc_f16(p.k);
      const uint32_t sbo = kt * 16;
      const uint32_t a0 = smem_u32(s_a), bb0 = smem_u32(s_b);
      uint32_t n = 0;
      bool ok = true;
      for (int64_t tile = t0; tile < p.n_tiles && ok; tile += tstride) {
        for (int bl = 0; bl < nbl; ++bl, ++n) {
          const uint32_t slot = n % p.slots, buf = n & 1;
          if (!tc_wait(bar.a_full + slot, (n / p.slots) & 1, s_abort)) { ok = false; break; }
          if (!tc_wait(bar.t_empty + buf, ((n >> 1) & 1) ^ 1, s_abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_tmem = tmem + buf * 256;
          const uint32_t a_addr = a0 + slot * a_slot_bytes;
          const uint32_t b_addr = bb0 + bl * b_blk_bytes;
          for (int j = 0; j < kt / 16; ++j) {
            tc_mma_f16(d_tmem, smem_desc(a_addr + j * 256, 128, sbo),
                       smem_desc(b_addr + j * 256, 128, sbo), idesc, j > 0 ? 1u : 0u);
          }
          tc_commit(bar.t_full + buf);
        }
      }
      // Every issued MMA has completed once its buffer's last commit fired.
      if (ok) {
        for (uint32_t q = (n >= 2 ? n - 2 : 0); q < n; ++q) {
          if (!tc_wait(bar.t_full + (q & 1), (q >> 1) & 1, s_abort)) break;
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- epilogue
    const int eg = warp >> 2;          // 0: even steps, 1: odd steps
    const int sub = warp & 3;          // TMEM lane quarter
    const int row = sub * 32 + lane;   // tile row of this thread
    const uint32_t tbase = tmem + ((uint32_t)(sub * 32) << 16) + eg * 256;
    const int nch = p.k / 32;
    uint32_t n = 0;
    bool ok = true;
    for (int64_t tile = t0; tile < p.n_tiles && ok; tile += tstride) {
      const int64_t r = tile * kTcRows + row;
      const bool valid = r < p.n_rows;
      int64_t g = 0, t = 0;
      if (valid) key_row_addr(p, r, g, t);
      for (int bl = 0; bl < nbl; ++bl, ++n) {
        if ((int)(n & 1) != eg) continue;
        const int b = b0 + bl;
        const uint32_t slot = n % p.slots;
        ok = __all_sync(0xffffffffu, tc_wait(bar.t_full + eg, (n >> 1) & 1, s_abort));
        if (!ok) break;
        tc_fence_after();
        const bool heavy = s_heavy[b] != 0;
        float s1 = __int_as_float(0x7f800000), s2 = s1;
        int c1chunk = 0;
        if (!heavy) {
          for (int ch = 0; ch < nch; ++ch) {
            uint32_t v[32];
            tc_ld32(tbase + ch * 32, v);
            tc_wait_ld();
            const float old = s1;
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const float a = __uint_as_float((v[j] & 0xFFFFFF00u) | (uint32_t)j);
              const float c = __uint_as_float((v[j + 1] & 0xFFFFFF00u) | (uint32_t)(j + 1));
              const float lo = fminf(a, c), hi = fmaxf(a, c);
              s2 = fmin3(s2, hi, fmaxf(s1, lo));
              s1 = fminf(s1, lo);
            }
            if (s1 != old) c1chunk = ch;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar.t_empty + eg);
        // acquire the producer's key norms (that phase has already completed)
        ok = __all_sync(0xffffffffu, tc_wait(bar.a_full + slot, (n / p.slots) & 1, s_abort));
        if (!ok) break;
        const float kn = s_kn[slot * kTcRows + row];
        __syncwarp();
        if (lane == 0) mbar_arrive(bar.a_empty + slot);
        int idx = 0;
        bool need = false;
        if (!heavy) {
          idx = c1chunk * 32 + (int)(__float_as_uint(s1) & 31u);
          const float sn = kn + s_cmax[bl];
          need = valid && !(s2 - s1 > sn * kTieRel && sn >= s_slo[bl] && sn <= s_shi[bl]);
        }
        uint32_t m = __ballot_sync(0xffffffffu, need);
        while (m) {
          const int src = __ffs(m) - 1;
          m &= m - 1;
          const int64_t rr = tile * kTcRows + sub * 32 + src;
          int bi;
          bi = exact_rescan<BD>(p, s_perm, rr, b, lane);
          if (lane == src) idx = bi;
        }
        if (valid) p.out_idx[g * p.igs + t * p.irs + b] = (uint8_t)idx;
      }
    }
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
// Returns SS_ERR_UNSUPPORTED when the tensor-core path does not apply.
int launch_vq_assign_tc(const void* keys, int key_dtype, int64_t n_groups, int64_t rpg,
                        int64_t kgs, int64_t krs, int d, const int32_t* perm,
                        const float* cents, int bd, int k, const uint8_t* heavy,
                        uint8_t* out_idx, int64_t igs, int64_t irs, uint16_t* out_heavy,
                        int64_t hgs, int64_t hrs, float* out_pt, int dist_mode,
                        cudaStream_t st) {
  const int es = key_dtype == SS_F32 ? 4 : 2;
  if (!(bd == 4 || bd == 8 || bd == 16)) return SS_ERR_UNSUPPORTED;
  if (k % 32 != 0 || k < 32 || k > 256) return SS_ERR_UNSUPPORTED;
  if (d > 128 || (d * es) % 16 != 0) return SS_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(keys) & 15) != 0) return SS_ERR_UNSUPPORTED;
  if (((kgs * es) & 15) != 0 || ((krs * es) & 15) != 0) return SS_ERR_UNSUPPORTED;
  const int nb = d / bd;
  const int kt = bd == 4 ? TcShape<4>::kKt : bd == 8 ? TcShape<8>::kKt : TcShape<16>::kKt;
  const uint32_t stage_stride = (uint32_t)(d * es + 4);
  const uint32_t stage_bytes = (kTcRows * stage_stride + 127) / 128 * 128;
  const uint32_t misc_bytes = 8 * 40 + 2048 + 4 * 32 * 4 + 256 + 16;
  const uint32_t b_blk = (uint32_t)k * kt * 2, a_slot = kTcRows * kt * 2;
  const uint32_t kn_slot = kTcRows * 4;
  const uint32_t limit = 227 * 1024;
  int slots = 6, gsize = 0;
  for (; slots >= 4; slots -= 2) {
    const uint32_t fixed = slots * (a_slot + kn_slot) + stage_bytes + misc_bytes + 1024;
    if (fixed < limit) gsize = (int)((limit - fixed) / b_blk);
    if (gsize >= 1) break;
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
  p.n_grp = n_grp; p.gsize = gsize; p.slots = slots;
  p.n_rows = n_groups * rpg;
  p.n_tiles = (p.n_rows + kTcRows - 1) / kTcRows;
  uint32_t off = 0;
  p.off_b = off; off += (uint32_t)gsize * b_blk;
  p.off_a = off; off += slots * a_slot;
  p.off_kn = off; off += slots * kn_slot;
  p.off_stage = off; off += stage_bytes;
  p.off_misc = off; off += misc_bytes;
  p.stage_stride = stage_stride;
  if (off > limit) return SS_ERR_UNSUPPORTED;
  // More than half an SM's shared memory: exactly one CTA (and one 512-column
  // TMEM allocation) per SM, so allocations never wait on each other.
  const uint32_t smem = off < 120 * 1024 ? 120 * 1024 : off;
  int per_grp = sm_count() / n_grp;
  if (per_grp < 1) per_grp = 1;
  if (per_grp > p.n_tiles) per_grp = (int)p.n_tiles;
  const int grid = per_grp * n_grp;
#define SS_LAUNCH_TC(BDV)                                                                   \
  case BDV:                                                                                 \
    cudaFuncSetAttribute(vq_assign_tc_kernel<BDV>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                         (int)smem);                                                        \
    vq_assign_tc_kernel<BDV><<<grid, kTcThreads, smem, st>>>(p);                            \
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
