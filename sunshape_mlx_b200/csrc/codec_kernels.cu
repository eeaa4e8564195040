// Block-VQ codec kernels: nearest-centroid assignment, k-means update,
// gather scores and reconstruction.
//
// Assignment reproduces the reference's CPU arithmetic exactly
// (codec.py:497-499): d = k - c and d*d are single float32 roundings and the
// sum over the block follows NumPy's pairwise order (for n < 8 a left-to-right
// sum; for 8 <= n <= 16 eight partial sums combined as ((0+1)+(2+3))+((4+5)+
// (6+7))). All float ops use explicit round-to-nearest intrinsics so the
// compiler cannot contract them into FMAs.
#include "common.cuh"
#include "vq_math.cuh"

namespace ss {
namespace {

constexpr int kAssignThreads = 512;
constexpr int kAssignRows = 32;  // rows per tile (one per lane)

struct AssignParams {
  const void* keys;
  int key_dtype;
  int64_t n_groups, rpg, kgs, krs;
  int d, nb, k;
  const int32_t* perm;
  const float* cents;
  const uint8_t* heavy;
  uint8_t* out_idx;
  int64_t igs, irs;
  uint16_t* out_heavy;
  int64_t hgs, hrs;
  float* out_pt;
  int dist_mode;
  int b_per_cta;  // blocks handled by one CTA (grid.y = ceil(nb / b_per_cta))
  // optional value rows copied (as f16) next to the keys: a cache append
  const void* vsrc;
  int vdt;
  int64_t vgs, vrs;
  uint16_t* vdst;
  int64_t vdgs, vdrs;
};

// Value rows of a cache append: rows [r0, r0 + n) of the (group, row) space,
// d elements each, converted to f16 (the cache's value dtype). Loads are
// issued in batches of 8 before their stores (the source and destination may
// alias as far as the compiler knows, which would otherwise serialize every
// element on a memory round trip); fp16 rows with 16-byte aligned strides
// move as 16-byte chunks.
__device__ __forceinline__ void copy_value_rows(const AssignParams& p, int64_t r0, int n,
                                                int tid, int nthr) {
  const int64_t n_rows = p.n_groups * p.rpg;
  const bool vec = p.vdt == SS_F16 && p.d % 8 == 0 &&
                   (reinterpret_cast<uintptr_t>(p.vsrc) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(p.vdst) & 15) == 0 && (p.vgs * 2) % 16 == 0 &&
                   (p.vrs * 2) % 16 == 0 && (p.vdgs * 2) % 16 == 0 && (p.vdrs * 2) % 16 == 0;
  if (vec) {
    const int cpr = p.d / 8;  // 16-byte chunks per row
    for (int e = tid; e < n * cpr; e += nthr) {
      const int rr = e / cpr, ch = e - rr * cpr;
      const int64_t r = r0 + rr;
      if (r >= n_rows) continue;
      const int64_t g = r / p.rpg, t = r - g * p.rpg;
      const uint4 v = *reinterpret_cast<const uint4*>(
          static_cast<const uint16_t*>(p.vsrc) + g * p.vgs + t * p.vrs + ch * 8);
      *reinterpret_cast<uint4*>(p.vdst + g * p.vdgs + t * p.vdrs + ch * 8) = v;
    }
    return;
  }
  for (int e0 = tid; e0 < n * p.d; e0 += 8 * nthr) {
    float x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = e0 + u * nthr;
      const int rr = e / p.d, j = e - rr * p.d;
      const int64_t r = r0 + rr;
      x[u] = 0.f;
      if (e < n * p.d && r < n_rows) {
        const int64_t g = r / p.rpg, t = r - g * p.rpg;
        x[u] = load_as_f32(p.vsrc, p.vdt, g * p.vgs + t * p.vrs + j);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = e0 + u * nthr;
      const int rr = e / p.d, j = e - rr * p.d;
      const int64_t r = r0 + rr;
      if (e < n * p.d && r < n_rows) {
        const int64_t g = r / p.rpg, t = r - g * p.rpg;
        p.vdst[g * p.vdgs + t * p.vdrs + j] = f2h(x[u]);
      }
    }
  }
}

__global__ void __launch_bounds__(256) copy_value_rows_small_kernel(AssignParams p) {
  copy_value_rows(p, (int64_t)blockIdx.x * 32, 32, threadIdx.x, 256);
}

// Bulk append of value rows: one thread per 8 consecutive elements of a row,
// one 16-byte load and store when the source is aligned f16.
__global__ void __launch_bounds__(256) copy_value_rows_kernel(AssignParams p, int vec) {
  const int per_row = p.d / 8;
  const int64_t n_rows = p.n_groups * p.rpg;
  const int64_t gid = (int64_t)blockIdx.x * 256 + threadIdx.x;
  const int64_t r = gid / per_row;
  if (r >= n_rows) return;
  const int j = static_cast<int>(gid - r * per_row) * 8;
  const int64_t g = r / p.rpg, t = r - g * p.rpg;
  uint16_t* dst = p.vdst + g * p.vdgs + t * p.vdrs + j;
  const int64_t so = g * p.vgs + t * p.vrs + j;
  if (vec) {
    *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(
        static_cast<const uint16_t*>(p.vsrc) + so));
    return;
  }
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = (uint32_t)f2h(load_as_f32(p.vsrc, p.vdt, so + 2 * i)) |
           ((uint32_t)f2h(load_as_f32(p.vsrc, p.vdt, so + 2 * i + 1)) << 16);
  *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
}

template <int BD>
__global__ void __launch_bounds__(kAssignThreads) vq_assign_kernel(AssignParams p) {
  extern __shared__ __align__(16) float sm[];
  const int b0 = blockIdx.y * p.b_per_cta;
  const int b1 = min(p.nb, b0 + p.b_per_cta);
  const int nbl = b1 - b0;
  float* s_c = sm;                                   // [nbl][k][BD]
  float* s_csq = s_c + (size_t)nbl * p.k * BD;       // [nbl][k] (expanded mode)
  float* s_k = s_csq + (size_t)nbl * p.k;            // [32][d + 1]
  uint8_t* s_idx = reinterpret_cast<uint8_t*>(s_k + kAssignRows * (p.d + 1));  // [32][nb]
  __shared__ int s_perm[1024];
  __shared__ uint8_t s_heavy[128];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < p.d; i += kAssignThreads) s_perm[i] = p.perm ? p.perm[i] : i;
  for (int i = tid; i < p.nb; i += kAssignThreads) s_heavy[i] = p.heavy ? p.heavy[i] : 0;
  const int nc = nbl * p.k * BD;
  const float* gc = p.cents + (size_t)b0 * p.k * BD;
  for (int i = tid; i < nc; i += kAssignThreads) s_c[i] = gc[i];
  __syncthreads();
  if (p.dist_mode == 1) {
    for (int i = tid; i < nbl * p.k; i += kAssignThreads) {
      float r[BD];
#pragma unroll
      for (int j = 0; j < BD; ++j) r[j] = __fmul_rn(s_c[i * BD + j], s_c[i * BD + j]);
      s_csq[i] = np_pairwise_sum<BD>(r);
    }
  }

  const int64_t n_rows = p.n_groups * p.rpg;
  const int64_t n_tiles = (n_rows + kAssignRows - 1) / kAssignRows;
  for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    const int64_t r0 = tile * kAssignRows;
    __syncthreads();  // previous tile's s_k / s_idx fully consumed
    // Load the permuted key tile as float32.
    for (int e = tid; e < kAssignRows * p.d; e += kAssignThreads) {
      const int rr = e / p.d, j = e - rr * p.d;
      const int64_t r = r0 + rr;
      float v = 0.f;
      if (r < n_rows) {
        const int64_t g = r / p.rpg, t = r - g * p.rpg;
        const int64_t off = g * p.kgs + t * p.krs + s_perm[j];
        v = load_as_f32(p.keys, p.key_dtype, off);
      }
      s_k[rr * (p.d + 1) + j] = v;
    }
    __syncthreads();
    const int64_t r = r0 + lane;
    const bool valid = r < n_rows;
    for (int bl = warp; bl < nbl; bl += kAssignThreads / 32) {
      const int b = b0 + bl;
      float kk[BD];
#pragma unroll
      for (int j = 0; j < BD; ++j) kk[j] = s_k[lane * (p.d + 1) + b * BD + j];
      int best_i = 0;
      if (!s_heavy[b]) {
        const float* cb = s_c + (size_t)bl * p.k * BD;
        float best = 0.f;
        if (p.dist_mode == 0) {
          best = dist_direct<BD>(kk, cb);
#pragma unroll 4
          for (int c = 1; c < p.k; ++c) {
            const float dd = dist_direct<BD>(kk, cb + c * BD);
            if (dd < best) { best = dd; best_i = c; }
          }
        } else {
          // ||x||^2 + ||c||^2 - (2x).c, as NumPy/BLAS evaluate codec.py:88-90
          float r2[BD];
          float x2[BD];
#pragma unroll
          for (int j = 0; j < BD; ++j) {
            r2[j] = __fmul_rn(kk[j], kk[j]);
            x2[j] = __fmul_rn(2.0f, kk[j]);
          }
          const float xsq = np_pairwise_sum<BD>(r2);
          const float* csq = s_csq + (size_t)bl * p.k;
          for (int c = 0; c < p.k; ++c) {
            float dot = 0.f;
#pragma unroll
            for (int j = 0; j < BD; ++j) dot = __fmaf_rn(x2[j], cb[c * BD + j], dot);
            const float dd = __fsub_rn(__fadd_rn(xsq, csq[c]), dot);
            if (c == 0 || dd < best) { best = dd; best_i = c; }
          }
        }
      } else if (valid) {
        const int64_t g = r / p.rpg, t = r - g * p.rpg;
        if (p.out_heavy) {
          int hpos = 0;
          for (int bb = 0; bb < b; ++bb) hpos += s_heavy[bb];
          uint16_t* dst = p.out_heavy + g * p.hgs + t * p.hrs + hpos * BD;
#pragma unroll
          for (int j = 0; j < BD; ++j) dst[j] = f2h(kk[j]);
        }
        if (p.out_pt) {
          float* dst = p.out_pt + r * (int64_t)p.nb * BD + b * BD;
#pragma unroll
          for (int j = 0; j < BD; ++j) dst[j] = kk[j];
        }
      }
      s_idx[lane * p.nb + b] = static_cast<uint8_t>(best_i);
    }
    __syncthreads();
    for (int e = tid; e < kAssignRows * nbl; e += kAssignThreads) {
      const int rr = e / nbl, b = b0 + (e - rr * nbl);
      const int64_t rw = r0 + rr;
      if (rw < n_rows) {
        const int64_t g = rw / p.rpg, t = rw - g * p.rpg;
        p.out_idx[g * p.igs + t * p.irs + b] = s_idx[rr * p.nb + b];
      }
    }
  }
}

// Few rows (a decode step's append): one CTA per (32-row tile, block); warp w
// scores centroids [w*k/16, (w+1)*k/16) for the tile's rows (lane = row), and
// the 16 partial winners are reduced in warp order. Same result as the
// sequential reference loop: the first index whose distance is below all
// earlier ones, a NaN distance at index 0 keeps 0.
template <int BD>
__global__ void __launch_bounds__(kAssignThreads) vq_assign_small_kernel(AssignParams p) {
  __shared__ float s_best[16][32];
  __shared__ int s_bi[16][32];
  __shared__ float s_d0[32];
  const int b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (p.vdst && b == 0) copy_value_rows(p, (int64_t)blockIdx.x * kAssignRows, kAssignRows, tid,
                                        kAssignThreads);
  const int64_t n_rows = p.n_groups * p.rpg;
  const int64_t r = (int64_t)blockIdx.x * kAssignRows + lane;
  const bool valid = r < n_rows;
  int64_t g = 0, t = 0;
  if (valid) { g = r / p.rpg; t = r - g * p.rpg; }
  float kk[BD];
#pragma unroll
  for (int j = 0; j < BD; ++j) {
    const int col = b * BD + j;
    kk[j] = valid ? load_as_f32(p.keys, p.key_dtype, g * p.kgs + t * p.krs + (p.perm ? p.perm[col] : col))
                  : 0.f;
  }
  const bool heavy = p.heavy && p.heavy[b];
  // the block's centroids, staged once with coalesced loads: the loop below
  // then reads them from shared memory instead of one dependent global
  // load per centroid
  __shared__ __align__(16) float s_c[256 * 16];
  const float* cb = p.cents + (size_t)b * p.k * BD;
  if (!heavy) {
    for (int e = tid; e < p.k * BD; e += kAssignThreads) s_c[e] = __ldg(cb + e);
  }
  __syncthreads();
  if (heavy) {
    if (warp == 0 && valid) {
      if (p.out_heavy) {
        int hpos = 0;
        for (int bb = 0; bb < b; ++bb) hpos += p.heavy[bb] ? 1 : 0;
        uint16_t* dst = p.out_heavy + g * p.hgs + t * p.hrs + hpos * BD;
#pragma unroll
        for (int j = 0; j < BD; ++j) dst[j] = f2h(kk[j]);
      }
      if (p.out_pt) {
        float* dst = p.out_pt + r * (int64_t)p.nb * BD + b * BD;
#pragma unroll
        for (int j = 0; j < BD; ++j) dst[j] = kk[j];
      }
      p.out_idx[g * p.igs + t * p.irs + b] = 0;
    }
    return;
  }
  const int per = (p.k + 15) / 16;
  const int c0 = warp * per, c1 = min(p.k, c0 + per);
  float best = __int_as_float(0x7f800000);
  int bi = 0x7fffffff;
  for (int c = c0; c < c1; ++c) {
    const float* cc = s_c + c * BD;
    const float dd = p.dist_mode == 0 ? dist_direct<BD>(kk, cc) : dist_expanded<BD>(kk, cc);
    if (c == 0) s_d0[lane] = dd;
    if (dd < best) { best = dd; bi = c; }
  }
  s_best[warp][lane] = best;
  s_bi[warp][lane] = bi;
  __syncthreads();
  if (warp == 0 && valid) {
    float bv = s_best[0][lane];
    int bx = s_bi[0][lane];
    for (int w = 1; w < 16; ++w) {
      if (s_best[w][lane] < bv) { bv = s_best[w][lane]; bx = s_bi[w][lane]; }
    }
    const float d0 = s_d0[lane];
    const int idx = (d0 != d0 || bx == 0x7fffffff) ? 0 : bx;
    p.out_idx[g * p.igs + t * p.irs + b] = static_cast<uint8_t>(idx);
  }
}

// ------------------------------------------------------------------ k-means
// One thread per (block, centroid): scans all rows in order and accumulates
// the assigned ones with float32 adds (same order as np.add.at).
__global__ void kmeans_update_kernel(const float* data, int64_t n, int nb, int bd,
                                     const uint8_t* assign, const float* cin, float* cout,
                                     int k) {
  const int gid = blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= nb * k) return;
  const int b = gid / k, c = gid - b * k;
  float acc[16];
  for (int j = 0; j < bd; ++j) acc[j] = 0.f;
  double cnt = 0.0;
  const int d = nb * bd;
  for (int64_t i = 0; i < n; ++i) {
    if (assign[i * nb + b] == c) {
      const float* x = data + i * d + b * bd;
      for (int j = 0; j < bd; ++j) acc[j] = __fadd_rn(acc[j], x[j]);
      cnt += 1.0;
    }
  }
  float* dst = cout + (size_t)gid * bd;
  const float* src = cin + (size_t)gid * bd;
  for (int j = 0; j < bd; ++j) {
    dst[j] = cnt > 0.0 ? static_cast<float>(static_cast<double>(acc[j]) / cnt) : src[j];
  }
}

// Same result with one CTA per block: a stable counting sort of the rows by
// centroid (shared-memory histogram, then 32 rows per step with match-any
// ranks so each centroid's rows keep their order), then one thread per
// centroid sums its rows in that order.
constexpr int kKmThreads = 256;
constexpr int kKmMaxRowsSorted = 49152;  // row list in shared memory
__global__ void __launch_bounds__(kKmThreads) kmeans_update_sorted_kernel(
    const float* data, int n, int nb, int bd, const uint8_t* assign, const float* cin,
    float* cout, int k) {
  extern __shared__ int sm_km[];
  int* s_cnt = sm_km;          // [256]
  int* s_off = sm_km + 256;    // [256] running end offsets
  int* s_list = sm_km + 512;   // [n] row ids grouped by centroid, rows in order
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  for (int c = tid; c < 256; c += kKmThreads) s_cnt[c] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += kKmThreads) atomicAdd(&s_cnt[assign[(int64_t)i * nb + b]], 1);
  __syncthreads();
  if (tid < 32) {
    // exclusive scan of the 256 counts: 8 per lane
    int loc[8], sum = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) { loc[q] = sum; sum += s_cnt[lane * 8 + q]; }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int base = incl - sum;
#pragma unroll
    for (int q = 0; q < 8; ++q) s_off[lane * 8 + q] = base + loc[q];
    __syncwarp();
    const unsigned lt = (1u << lane) - 1u;
    for (int r0 = 0; r0 < n; r0 += 32) {
      const int i = r0 + lane;
      const int c = i < n ? (int)assign[(int64_t)i * nb + b] : 256 + lane;  // unique filler
      const unsigned same = __match_any_sync(0xffffffffu, c);
      if (i < n) s_list[s_off[c] + __popc(same & lt)] = i;
      __syncwarp();
      if (i < n && lane == 31 - __clz(same)) s_off[c] += __popc(same);
      __syncwarp();
    }
  }
  __syncthreads();
  const int d = nb * bd;
  for (int c = tid; c < k; c += kKmThreads) {
    const int end = s_off[c], cnt = s_cnt[c];
    float acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0.f;
    for (int q = end - cnt; q < end; ++q) {
      const float* x = data + (int64_t)s_list[q] * d + b * bd;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (j < bd) acc[j] = __fadd_rn(acc[j], x[j]);
      }
    }
    float* dst = cout + ((size_t)b * k + c) * bd;
    const float* src = cin + ((size_t)b * k + c) * bd;
    for (int j = 0; j < bd; ++j) {
      dst[j] = cnt > 0 ? static_cast<float>(static_cast<double>(acc[j]) / static_cast<double>(cnt))
                       : src[j];
    }
  }
}

// ------------------------------------------------------------------ scores
// grid.x over token tiles of 256, grid.y over query chunks of 8; the LUT of
// the chunk lives in shared memory.
constexpr int kScoreQ = 8;
__global__ void __launch_bounds__(256) vq_scores_kernel(const float* q, int nq, int d,
                                                        const float* cents, int bd, int k,
                                                        const float* lut_in, int nb,
                                                        const uint8_t* idx, int64_t t,
                                                        int64_t irs, float* out, int64_t os) {
  extern __shared__ float lut[];  // [kScoreQ][nb][k]
  const int q0 = blockIdx.y * kScoreQ;
  const int nql = min(kScoreQ, nq - q0);
  for (int e = threadIdx.x; e < nql * nb * k; e += blockDim.x) {
    if (lut_in) {
      lut[e] = lut_in[(size_t)q0 * nb * k + e];
      continue;
    }
    const int qi = e / (nb * k), rem = e - qi * nb * k, b = rem / k, c = rem - b * k;
    const float* qq = q + (int64_t)(q0 + qi) * d + b * bd;
    const float* cc = cents + ((size_t)b * k + c) * bd;
    float acc = 0.f;
    for (int j = 0; j < bd; ++j) acc = fmaf(qq[j], cc[j], acc);
    lut[e] = acc;
  }
  __syncthreads();
  const int64_t tok = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (tok >= t) return;
  const uint8_t* row = idx + tok * irs;
  for (int qi = 0; qi < nql; ++qi) {
    const float* l = lut + (size_t)qi * nb * k;
    float s = 0.f;
    for (int b = 0; b < nb; ++b) s += l[b * k + row[b]];
    out[(int64_t)(q0 + qi) * os + tok] = s;
  }
}

// ------------------------------------------------------------------ query x centroid table
// out[q][b][c] = sum_j q[q][b * bd + j] * C[b][c][j] (fused multiply-adds in j
// order). One thread per (q, b, c): consecutive threads write consecutive
// centroids, so the table is written coalesced.
__global__ void __launch_bounds__(256) query_centroid_dots_kernel(const float* q, int64_t nq, int d,
                                                                  const float* cents, int bd, int k,
                                                                  float* out) {
  const int nb = d / bd;
  const int64_t n = nq * nb * k;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t qi = e / ((int64_t)nb * k);
    const int rem = static_cast<int>(e - qi * nb * k);
    const int b = rem / k, c = rem - b * k;
    const float* qq = q + qi * d + b * bd;
    const float* cc = cents + ((size_t)b * k + c) * bd;
    float acc = 0.f;
    for (int j = 0; j < bd; ++j) acc = fmaf(__ldg(qq + j), __ldg(cc + j), acc);
    out[e] = acc;
  }
}

// ------------------------------------------------------------------ row transform
// out[r][j] = sum_i x[r][i] * m[i][j] (fused multiply-adds in i order), the
// rotations of rotated-mode keys and of the TurboQuant fp16 tail. A CTA
// holds m (d x d f32) and a tile of kRotRows rows in shared memory; thread
// (column j, row group) accumulates kRotRows * blockDim / d rows.
constexpr int kRotRows = 64;
__global__ void __launch_bounds__(256) rotate_rows_kernel(const float* x, int64_t rows, int d,
                                                          int64_t xs, const float* m, void* out,
                                                          int odt, int64_t os) {
  extern __shared__ float rsm[];
  float* sm_m = rsm;              // [d][d]
  float* sm_x = rsm + d * d;      // [kRotRows][d]
  const int64_t r0 = (int64_t)blockIdx.x * kRotRows;
  const int nr = rows - r0 < kRotRows ? static_cast<int>(rows - r0) : kRotRows;
  for (int e = threadIdx.x; e < d * d; e += blockDim.x) sm_m[e] = m[e];
  for (int e = threadIdx.x; e < nr * d; e += blockDim.x) {
    const int rr = e / d, i = e - rr * d;
    sm_x[e] = x[(r0 + rr) * xs + i];
  }
  __syncthreads();
  const int j = threadIdx.x % d;
  const int groups = blockDim.x / d;
  const int g = threadIdx.x / d;
  if (g >= groups) return;
  constexpr int kMaxRpt = kRotRows;  // rows per thread at d = blockDim (upper bound)
  const int rpt = kRotRows / groups;
  float acc[kMaxRpt / 2];
  for (int base = 0; base < rpt; base += kMaxRpt / 2) {
    const int n = min(kMaxRpt / 2, rpt - base);
#pragma unroll
    for (int q = 0; q < kMaxRpt / 2; ++q) acc[q] = 0.f;
    for (int i = 0; i < d; ++i) {
      const float mv = sm_m[i * d + j];
#pragma unroll
      for (int q = 0; q < kMaxRpt / 2; ++q)
        if (q < n) acc[q] = fmaf(sm_x[(g * rpt + base + q) * d + i], mv, acc[q]);
    }
    for (int q = 0; q < n; ++q) {
      const int rr = g * rpt + base + q;
      if (rr < nr) store_from_f32(out, odt, (r0 + rr) * os + j, acc[q]);
    }
  }
}

// ------------------------------------------------------------------ dequant
__global__ void vq_dequant_kernel(const uint8_t* idx, int64_t n_groups, int64_t rpg,
                                  int64_t igs, int64_t irs, const float* cents, int d, int bd,
                                  int k, const int32_t* inv_perm, const uint8_t* heavy,
                                  const uint16_t* hv, int64_t hgs, int64_t hrs, void* out,
                                  int odt, int64_t ogs, int64_t ors) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = n_groups * rpg * d;
  if (e >= total) return;
  const int64_t r = e / d;
  const int j = static_cast<int>(e - r * d);  // output (original-basis) column
  const int64_t g = r / rpg, t = r - g * rpg;
  const int src = inv_perm ? inv_perm[j] : j;  // codec-space column
  const int b = src / bd, w = src - b * bd;
  float v;
  if (heavy && heavy[b]) {
    int hpos = 0;
    for (int bb = 0; bb < b; ++bb) hpos += heavy[bb];
    v = hv ? h2f(hv[g * hgs + t * hrs + hpos * bd + w]) : 0.f;
  } else {
    const int c = idx[g * igs + t * irs + b];
    v = cents[((size_t)b * k + c) * bd + w];
  }
  store_from_f32(out, odt, g * ogs + t * ors + j, v);
}

}  // namespace
}  // namespace ss

namespace ss {
int launch_vq_assign_tc(const void* keys, int key_dtype, int64_t n_groups, int64_t rpg,
                        int64_t kgs, int64_t krs, int d, const int32_t* perm,
                        const float* cents, int bd, int k, const uint8_t* heavy,
                        uint8_t* out_idx, int64_t igs, int64_t irs, uint16_t* out_heavy,
                        int64_t hgs, int64_t hrs, float* out_pt, int dist_mode,
                        cudaStream_t st);
}  // namespace ss

using namespace ss;

namespace {
// 0 = automatic, 1 = CUDA-core kernel only, 2 = tensor-core kernel required.
int g_assign_path = 0;
// Below this many rows the CUDA-core kernel has the lower latency.
constexpr int64_t kTcMinRows = 16384;
// At most this many rows: the (row tile x block) kernel for small appends.
constexpr int64_t kSmallRows = 4096;
}  // namespace

extern "C" {

int ss_set_assign_path(int path) {
  SS_REQUIRE(path >= 0 && path <= 2, "ss_set_assign_path: path must be 0, 1 or 2");
  g_assign_path = path;
  return SS_OK;
}

int ss_vq_assign(const void* keys, int key_dtype, int64_t n_groups, int64_t rows_per_group,
                 int64_t key_group_stride, int64_t key_row_stride, int d, const int32_t* perm,
                 const float* centroids, int bd, int k, const uint8_t* heavy, uint8_t* out_idx,
                 int64_t idx_group_stride, int64_t idx_row_stride, uint16_t* out_heavy,
                 int64_t heavy_group_stride, int64_t heavy_row_stride, float* out_pt,
                 int dist_mode, void* stream) {
  SS_REQUIRE(keys && centroids && out_idx, "ss_vq_assign: null pointer");
  SS_REQUIRE(d > 0 && d <= 1024 && bd > 0 && d % bd == 0, "ss_vq_assign: bad d / bd");
  SS_REQUIRE(k >= 1 && k <= 256, "ss_vq_assign: k must be in [1, 256] (uint8 indices)");
  SS_REQUIRE(d / bd <= 128, "ss_vq_assign: at most 128 blocks");
  SS_REQUIRE(key_dtype >= SS_F32 && key_dtype <= SS_BF16, "ss_vq_assign: bad key dtype");
  SS_REQUIRE(dist_mode == 0 || dist_mode == 1, "ss_vq_assign: bad dist_mode");
  count_dispatch("ss_vq_assign");
  if (n_groups <= 0 || rows_per_group <= 0) return SS_OK;
  if (g_assign_path == 2 || (g_assign_path == 0 && n_groups * rows_per_group >= kTcMinRows)) {
    const int rc = launch_vq_assign_tc(keys, key_dtype, n_groups, rows_per_group, key_group_stride,
                                       key_row_stride, d, perm, centroids, bd, k, heavy, out_idx,
                                       idx_group_stride, idx_row_stride, out_heavy,
                                       heavy_group_stride, heavy_row_stride, out_pt, dist_mode,
                                       as_stream(stream));
    if (rc != SS_ERR_UNSUPPORTED) return rc;
    if (g_assign_path == 2) {
      return fail(SS_ERR_UNSUPPORTED,
                  "ss_vq_assign: the tensor-core path needs bd in {4,8,16}, k a multiple of 64, "
                  "d <= 128 and 16-byte aligned key rows");
    }
  }
  AssignParams p{keys, key_dtype, n_groups, rows_per_group, key_group_stride, key_row_stride,
                 d, d / bd, k, perm, centroids, heavy, out_idx, idx_group_stride,
                 idx_row_stride, out_heavy, heavy_group_stride, heavy_row_stride, out_pt,
                 dist_mode, 0};
  if (n_groups * rows_per_group <= kSmallRows && g_assign_path != 2) {
    // a decode step's append: spread (row tile, block) pairs over the SMs
    const dim3 grid_s(static_cast<unsigned>((n_groups * rows_per_group + kAssignRows - 1) / kAssignRows),
                      static_cast<unsigned>(p.nb));
    cudaStream_t sst = as_stream(stream);
    switch (bd) {
      case 2: vq_assign_small_kernel<2><<<grid_s, kAssignThreads, 0, sst>>>(p); break;
      case 4: vq_assign_small_kernel<4><<<grid_s, kAssignThreads, 0, sst>>>(p); break;
      case 8: vq_assign_small_kernel<8><<<grid_s, kAssignThreads, 0, sst>>>(p); break;
      case 16: vq_assign_small_kernel<16><<<grid_s, kAssignThreads, 0, sst>>>(p); break;
      default: return fail(SS_ERR_UNSUPPORTED, "ss_vq_assign: block_dim must be 2, 4, 8 or 16");
    }
    return check_launch("ss_vq_assign (small)");
  }
  // Blocks per CTA so that the centroid slice stays within ~160 KB of smem.
  const size_t per_block = (size_t)k * bd * 4 + (size_t)k * 4;
  int bpc = static_cast<int>((160 * 1024) / per_block);
  bpc = bpc < 1 ? 1 : (bpc > p.nb ? p.nb : bpc);
  p.b_per_cta = bpc;
  const size_t smem = per_block * bpc + (size_t)kAssignRows * (d + 1) * 4 +
                      (size_t)kAssignRows * p.nb;
  const int64_t n_tiles = (n_groups * rows_per_group + kAssignRows - 1) / kAssignRows;
  const int gy = (p.nb + bpc - 1) / bpc;
  int gx = sm_count() / gy;
  if (gx < 1) gx = 1;
  if (gx > n_tiles) gx = static_cast<int>(n_tiles);
  dim3 grid(gx, gy);
  cudaStream_t st = as_stream(stream);
#define SS_LAUNCH_ASSIGN(BDV)                                                               \
  case BDV:                                                                                 \
    cudaFuncSetAttribute(vq_assign_kernel<BDV>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                         (int)smem);                                                       \
    vq_assign_kernel<BDV><<<grid, kAssignThreads, smem, st>>>(p);                           \
    break;
  switch (bd) {
    SS_LAUNCH_ASSIGN(2)
    SS_LAUNCH_ASSIGN(4)
    SS_LAUNCH_ASSIGN(8)
    SS_LAUNCH_ASSIGN(16)
    default:
      return fail(SS_ERR_UNSUPPORTED, "ss_vq_assign: block_dim must be 2, 4, 8 or 16");
  }
#undef SS_LAUNCH_ASSIGN
  return check_launch("ss_vq_assign");
}

int ss_cache_append(const ss_append_args* a, void* stream) {
  SS_REQUIRE(a && a->keys && a->values && a->idx && a->v && a->centroids,
             "ss_cache_append: null pointer");
  SS_REQUIRE(a->value_dtype >= SS_F32 && a->value_dtype <= SS_BF16,
             "ss_cache_append: bad value dtype");
  const int64_t rows = a->n_groups * a->rows;
  if (a->n_groups <= 0 || a->rows <= 0) return SS_OK;
  const bool small = rows <= kSmallRows && g_assign_path != 2 &&
                     (a->bd == 2 || a->bd == 4 || a->bd == 8 || a->bd == 16);
  if (!small) {
    // bulk append (prefill): the assignment dispatch of ss_vq_assign, then the value rows
    const int rc = ss_vq_assign(a->keys, a->key_dtype, a->n_groups, a->rows, a->key_group_stride,
                                a->key_row_stride, a->d, a->perm, a->centroids, a->bd, a->k,
                                a->heavy, a->idx, a->idx_group_stride, a->idx_row_stride,
                                a->kheavy, a->kheavy_group_stride, a->kheavy_row_stride, nullptr,
                                0, stream);
    if (rc != SS_OK) return rc;
  }
  SS_REQUIRE(a->d > 0 && a->d <= 1024 && a->d % a->bd == 0 && a->d / a->bd <= 128,
             "ss_cache_append: bad d / bd");
  SS_REQUIRE(a->k >= 1 && a->k <= 256, "ss_cache_append: k must be in [1, 256]");
  SS_REQUIRE(a->key_dtype >= SS_F32 && a->key_dtype <= SS_BF16, "ss_cache_append: bad key dtype");
  AssignParams p{a->keys, a->key_dtype, a->n_groups, a->rows, a->key_group_stride,
                 a->key_row_stride, a->d, a->d / a->bd, a->k, a->perm, a->centroids, a->heavy,
                 a->idx, a->idx_group_stride, a->idx_row_stride, a->kheavy,
                 a->kheavy_group_stride, a->kheavy_row_stride, nullptr, 0, 0,
                 a->values, a->value_dtype, a->value_group_stride, a->value_row_stride, a->v,
                 a->v_group_stride, a->v_row_stride};
  cudaStream_t st = as_stream(stream);
  const unsigned tiles = static_cast<unsigned>((rows + kAssignRows - 1) / kAssignRows);
  if (!small) {
    if (a->d % 8 == 0 && reinterpret_cast<uintptr_t>(a->v) % 16 == 0 &&
        (a->v_group_stride * 2) % 16 == 0 && (a->v_row_stride * 2) % 16 == 0) {
      const int es = a->value_dtype == SS_F32 ? 4 : 2;
      const int vec = a->value_dtype == SS_F16 && reinterpret_cast<uintptr_t>(a->values) % 16 == 0 &&
                      (a->value_group_stride * es) % 16 == 0 && (a->value_row_stride * es) % 16 == 0;
      const int64_t n = rows * (a->d / 8);
      copy_value_rows_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(p, vec);
    } else {
      copy_value_rows_small_kernel<<<tiles, 256, 0, st>>>(p);
    }
    return check_launch("ss_cache_append (values)");
  }
  count_dispatch("ss_cache_append");
  const dim3 grid_s(tiles, static_cast<unsigned>(p.nb));
  switch (a->bd) {
    case 2: vq_assign_small_kernel<2><<<grid_s, kAssignThreads, 0, st>>>(p); break;
    case 4: vq_assign_small_kernel<4><<<grid_s, kAssignThreads, 0, st>>>(p); break;
    case 8: vq_assign_small_kernel<8><<<grid_s, kAssignThreads, 0, st>>>(p); break;
    default: vq_assign_small_kernel<16><<<grid_s, kAssignThreads, 0, st>>>(p); break;
  }
  return check_launch("ss_cache_append");
}

int ss_kmeans_update(const float* data, int64_t n, int nb, int bd, const uint8_t* assign,
                     const float* cents_in, float* cents_out, int k, void* stream) {
  SS_REQUIRE(data && assign && cents_in && cents_out, "ss_kmeans_update: null pointer");
  SS_REQUIRE(cents_in != cents_out, "ss_kmeans_update: cents_in and cents_out alias");
  SS_REQUIRE(bd >= 1 && bd <= 16 && nb >= 1 && k >= 1 && k <= 256, "ss_kmeans_update: bad dims");
  count_dispatch("ss_kmeans_update");
  if (n <= kKmMaxRowsSorted) {
    const size_t smem = (512 + (size_t)n) * sizeof(int);
    cudaFuncSetAttribute(kmeans_update_sorted_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    kmeans_update_sorted_kernel<<<nb, kKmThreads, smem, as_stream(stream)>>>(
        data, static_cast<int>(n), nb, bd, assign, cents_in, cents_out, k);
    return check_launch("ss_kmeans_update");
  }
  const int threads = 128;
  const int blocks = (nb * k + threads - 1) / threads;
  kmeans_update_kernel<<<blocks, threads, 0, as_stream(stream)>>>(data, n, nb, bd, assign,
                                                                   cents_in, cents_out, k);
  return check_launch("ss_kmeans_update");
}

int ss_vq_scores(const float* q, int nq, int d, const float* centroids, int bd, int k,
                 const uint8_t* idx, int64_t t, int64_t idx_row_stride, float* out,
                 int64_t out_stride, void* stream) {
  SS_REQUIRE(q && centroids && out && (idx || t == 0), "ss_vq_scores: null pointer");
  SS_REQUIRE(bd > 0 && d % bd == 0 && k >= 1 && k <= 256, "ss_vq_scores: bad dims");
  const size_t smem = (size_t)kScoreQ * (d / bd) * k * 4;
  SS_REQUIRE(smem <= 200 * 1024, "ss_vq_scores: lookup table too large for shared memory");
  count_dispatch("ss_vq_scores");
  if (nq <= 0 || t <= 0) return SS_OK;
  cudaFuncSetAttribute(vq_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(static_cast<unsigned>((t + 255) / 256), (nq + kScoreQ - 1) / kScoreQ);
  vq_scores_kernel<<<grid, 256, smem, as_stream(stream)>>>(q, nq, d, centroids, bd, k, nullptr,
                                                           d / bd, idx, t, idx_row_stride, out,
                                                           out_stride);
  return check_launch("ss_vq_scores");
}

int ss_query_centroid_dots(const float* q, int64_t nq, int d, const float* centroids, int bd,
                           int k, float* out, void* stream) {
  SS_REQUIRE(q && centroids && out, "ss_query_centroid_dots: null pointer");
  SS_REQUIRE(nq >= 0 && bd > 0 && d % bd == 0 && k >= 1 && k <= 256,
             "ss_query_centroid_dots: bad dims");
  count_dispatch("ss_query_centroid_dots");
  const int64_t n = nq * (d / bd) * k;
  if (n == 0) return SS_OK;
  int64_t blocks = (n + 255) / 256;
  if (blocks > (int64_t)sm_count() * 16) blocks = (int64_t)sm_count() * 16;
  query_centroid_dots_kernel<<<static_cast<unsigned>(blocks), 256, 0, as_stream(stream)>>>(
      q, nq, d, centroids, bd, k, out);
  return check_launch("ss_query_centroid_dots");
}

int ss_rotate_rows(const float* x, int64_t rows, int d, int64_t x_row_stride, const float* m,
                   void* out, int out_dtype, int64_t out_row_stride, void* stream) {
  SS_REQUIRE(x && m && out, "ss_rotate_rows: null pointer");
  SS_REQUIRE(d >= 1 && d <= 128 && 256 % d == 0 && rows >= 0,
             "ss_rotate_rows: d must be a power of two <= 128");
  count_dispatch("ss_rotate_rows");
  if (rows == 0) return SS_OK;
  const size_t smem = ((size_t)d * d + (size_t)kRotRows * d) * sizeof(float);
  cudaFuncSetAttribute(rotate_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  rotate_rows_kernel<<<static_cast<unsigned>((rows + kRotRows - 1) / kRotRows), 256, smem,
                       as_stream(stream)>>>(x, rows, d, x_row_stride, m, out, out_dtype,
                                            out_row_stride);
  return check_launch("ss_rotate_rows");
}

int ss_vq_scores_lut(const float* qdots, int nq, int nb, int k, const uint8_t* idx, int64_t t,
                     int64_t idx_row_stride, float* out, int64_t out_stride, void* stream) {
  SS_REQUIRE(qdots && out && (idx || t == 0), "ss_vq_scores_lut: null pointer");
  SS_REQUIRE(nb >= 1 && k >= 1 && k <= 256, "ss_vq_scores_lut: bad dims");
  const size_t smem = (size_t)kScoreQ * nb * k * 4;
  SS_REQUIRE(smem <= 200 * 1024, "ss_vq_scores_lut: lookup table too large for shared memory");
  count_dispatch("ss_vq_scores_lut");
  if (nq <= 0 || t <= 0) return SS_OK;
  cudaFuncSetAttribute(vq_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(static_cast<unsigned>((t + 255) / 256), (nq + kScoreQ - 1) / kScoreQ);
  vq_scores_kernel<<<grid, 256, smem, as_stream(stream)>>>(nullptr, nq, 0, nullptr, 1, k, qdots,
                                                           nb, idx, t, idx_row_stride, out,
                                                           out_stride);
  return check_launch("ss_vq_scores_lut");
}

int ss_vq_dequant(const uint8_t* idx, int64_t n_groups, int64_t rows_per_group,
                  int64_t idx_group_stride, int64_t idx_row_stride, const float* centroids,
                  int d, int bd, int k, const int32_t* inv_perm, const uint8_t* heavy,
                  const uint16_t* heavy_vals, int64_t heavy_group_stride,
                  int64_t heavy_row_stride, void* out, int out_dtype, int64_t out_group_stride,
                  int64_t out_row_stride, void* stream) {
  SS_REQUIRE(idx && centroids && out, "ss_vq_dequant: null pointer");
  SS_REQUIRE(bd > 0 && d % bd == 0 && k >= 1 && k <= 256, "ss_vq_dequant: bad dims");
  count_dispatch("ss_vq_dequant");
  const int64_t total = n_groups * rows_per_group * d;
  if (total <= 0) return SS_OK;
  const int threads = 256;
  vq_dequant_kernel<<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0,
                      as_stream(stream)>>>(
      idx, n_groups, rows_per_group, idx_group_stride, idx_row_stride, centroids, d, bd, k,
      inv_perm, heavy, heavy_vals, heavy_group_stride, heavy_row_stride, out, out_dtype,
      out_group_stride, out_row_stride);
  return check_launch("ss_vq_dequant");
}

}  // extern "C"
