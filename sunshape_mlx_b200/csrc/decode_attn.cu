// Fused SunShape attention over the compressed KV cache (decode and
// multi-query / causal prefill), one launch for the whole (B, Hq, Tq) output.
//
// Work decomposition. A "unit" is one (batch, kv-head) pair together with a
// group of up to R query rows of that kv-head (GQA repeats x query tokens).
// Each unit's token stream is cut into 128-token tiles (64 when R = 8):
// compressed tiles first, then tiles of the hybrid cache's fp16 tail. The
// flattened (unit, tile) sequence is split into equal contiguous ranges, one
// per persistent CTA (one CTA per SM), so every SM streams the same number
// of bytes regardless of batch/head counts. A CTA that covers a unit only
// partly writes an unnormalised (o, m, l) partial; the last CTA to finish a
// unit (self-resetting arrival counter) merges the partials by log-sum-exp.
//
// Inside a CTA: warp 8 is the producer. It streams the uint8 index tile with
// a 1-D bulk copy and the fp16 value tile with two 2-D-box tensor copies
// (128-byte swizzle, so the consumers' ldmatrix reads are conflict-free) into
// a ring of mbarrier-tracked stages. Warps 0-7 consume:
//   1. scores: each token's sum_b LUT[b][idx_b][r] (the query x centroid
//      table of every row of the unit, fp32, in shared memory), plus exact
//      dot products for mixed-precision heavy blocks and fp16 tail keys;
//   2. online softmax per row with a tile-wide max;
//   3. P.V on the tensor cores: O^T(dims x rows) += V^T(dims x tokens) .
//      P(tokens x rows) with mma.m16n8k16 (fp16 in, fp32 accumulate).
// Quantized values are first decoded (levels * scale + zero) into an fp16
// tile in the same swizzled layout and then take the same MMA path.
#include <algorithm>
#include <type_traits>
#include <cfloat>
#include <mutex>
#include <string>

#include "common.cuh"
#include "vq_math.cuh"

namespace ss {
namespace {

// Consumer warps per CTA (CW, a kernel template parameter): 8 with 4 stages
// of 128 tokens, or 12 with 6 stages when the stage is small (quantized
// values); one producer warp follows them.
constexpr int kLutThreads = 256;  // table kernel block size
constexpr int kMaxStages = 8;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // default bound of a barrier wait (2 s)
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeParams {
  // shapes
  int b, hq, hkv, tq, d, nb, bd, k, nrep, n_heavy;
  int R, tile, n_rg, n_ct, n_tt, tpu;
  int64_t tc, ttail, total_tiles, n_units;
  int grid, stages, stage_shift, max_cov;  // stages: a multiple of the tile groups
  int w_unit;                              // schedule cost of a unit boundary, in tiles
  // queries
  const void* q;
  int qdt;
  int64_t q_sb, q_sh, q_st;
  float scale;
  // codec
  const int32_t* perm;
  const float* rot_k;
  const float* cents;
  const uint8_t* heavy;
  // keys
  const uint8_t* idx;
  int64_t idx_ps;
  const uint16_t* kheavy;
  int64_t kh_ps;
  // values
  int vfmt;
  int64_t v_ps;  // fp16 V pair stride (elements), only for the byte count
  const uint32_t* vq;
  int64_t vq_ps;
  int v_bits, v_group, v_words, v_groups;
  int v_gshift;              // log2(v_group) when a power of two, else -1
  int vdec;                  // compressed value tiles: 0 fp16 (MMA straight from the
                             // stage), 1 2-bit fast decoder, 2 block-VQ, 3 generic
  const void* vs;
  int vs_dt;
  int64_t vs_ps;
  const float* vz;
  int64_t vz_ps;
  float levels[16];
  const float* v_rot;
  const uint8_t* vidx;       // SS_V_VQ: u8 rows v_nb
  int64_t vi_ps;
  const uint16_t* vcents;    // SS_V_VQ: f16 [v_nb][v_k][v_bd]
  int v_bd, v_k, v_nb;
  uint32_t v_tile_bytes;     // stage bytes of one tile's value stream (quantized / VQ)
  // tail
  const uint16_t* k_tail;
  const uint16_t* v_tail;
  int64_t tail_ps;
  // masking
  int causal;
  const float* mask;
  int64_t mask_stride;
  int mask_mode;
  // output
  void* out;
  int odt;
  int64_t o_sb, o_sh, o_st;
  float* part_out;  // non-null: write (o, m, l) rows instead of the output
  // workspace
  int* err;
  int* sink;                // process error sink (host word) or null
  uint64_t wait_ns;         // bound of every barrier wait
  int64_t skip_tile;        // test hook: tile whose copies are never issued (-1: none)
  // fused cache append (app_rows > 0): the newest app_rows tokens of every pair
  const void* app_k;
  const void* app_v;
  int app_dt;
  int64_t app_kps, app_krs, app_vps, app_vrs, app_rows;
  int app_groups;           // 8-row append CTAs per key block
  int lut_groups;           // table CTAs per key block (grid.y below the append CTAs)
  uint16_t* v_w;            // fp16 value stream (append writes)
  int* counters;
  float* slots;
  float* lut_g;             // per-unit query x centroid tables [unit][nb][k][R]
  uint32_t lut_unit_bytes;
  // shared-memory carve-up (bytes from the 1024-aligned base)
  uint32_t off_stage, stage_bytes, off_idx, off_aux, off_vdq, off_lut, off_p, off_misc, off_vtab;
  uint32_t off_plo;  // 8-row units: per-warp lo-half P slices (0: in the query rows of Misc)
};

// Tokens per consumer-warp slice (one per lane). With 128-token tiles this
// gives two tile groups of four warps, so four stages double-buffer each group.
__host__ __device__ constexpr int slice_tokens(int) { return 32; }

__device__ __forceinline__ uint32_t pack_halves2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// Maximum of v over the warp (NaN inputs ignored, as fmaxf does).
__device__ __forceinline__ float warp_max_f32(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

// 2^x with the SFU approximation (ex2.approx.ftz): |rel err| < 2^-22.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Static schedule. CTA k owns the tiles [start(k), start(k + 1)) of the
// (unit, tile) sequence. A tile costs 1 and every unit boundary costs w more
// (the merge, cross-CTA publish and table reload at a unit end), so ranges
// are equal in cost c(t) = t + w * floor(t / tpu), not in tiles; a CTA whose
// range crosses a unit boundary gets about w fewer tiles.
struct Sched {
  int64_t total, tpu, w, cost;  // cost = c(total - 1) + 1
  int grid;
};
__host__ __device__ inline Sched make_sched(int64_t total, int64_t tpu, int64_t w, int grid) {
  Sched s{total, tpu, w, total + w * (total / tpu - 1), grid};
  return s;
}
// smallest t with c(t) * grid >= k * cost
__host__ __device__ inline int64_t range_start(const Sched& s, int64_t k) {
  if (k >= s.grid) return s.total;
  const int64_t y = k * s.cost;
  const int64_t pg = (s.tpu + s.w) * s.grid;
  const int64_t j = y / pg;
  const int64_t x = (y - j * pg + s.grid - 1) / s.grid;
  const int64_t t = x < s.tpu ? j * s.tpu + x : (j + 1) * s.tpu;
  return t < s.total ? t : s.total;
}
// the CTA whose range holds tile t
__host__ __device__ inline int64_t cta_of(const Sched& s, int64_t t) {
  return (t + s.w * (t / s.tpu)) * s.grid / s.cost;
}

// Address of the 16-byte chunk holding V[tok][dim..dim+7] in a swizzled tile
// made of (d / 64) boxes of `tile` rows x 128 bytes.
__device__ __forceinline__ uint32_t vtile_addr(uint32_t base, int tile, int tok, int dim) {
  const int box = dim >> 6;
  const int chunk = (dim & 63) >> 3;
  return base + box * (tile * 128) + tok * 128 + ((chunk ^ (tok & 7)) << 4);
}

struct Misc {  // small shared-memory state
  float qo[8][128];     // scaled queries, original basis
  float qc[8][128];     // scaled queries, codec space
  float mrow[8], lrow[8];
  float levels[16];
  alignas(128) float2 lvpair[16];  // 2-bit values: levels of the two codes of each nibble
  int heavy_pos[32];
  uint8_t is_heavy[128];
  int is_last;
  int abort;
};

// Scaled query rows of a unit in the original basis: qo[r] = dtype(q * scale)
// (attention.py:208) for row r = (GQA repeat, query token) of group rg.
__device__ __forceinline__ void unit_query_rows(const DecodeParams& p, float (*qo)[128], int rg,
                                                int bb, int hh, int tid, int nthr) {
  const float sc = round_to(p.scale, p.qdt);
  const int rows_valid = p.nrep * p.tq;
  for (int e = tid; e < p.R * p.d; e += nthr) {
    const int r = e / p.d, j = e - r * p.d;
    const int rr = rg * p.R + r;
    float v = 0.f;
    if (rr < rows_valid) {
      const int rep = rr / p.tq, tqi = rr - rep * p.tq;
      const int qh = hh * p.nrep + rep;
      const float x = load_as_f32(p.q, p.qdt, bb * p.q_sb + qh * p.q_sh + tqi * p.q_st + j);
      v = round_to(x * sc, p.qdt);
    }
    qo[r][j] = v;
  }
}

// The same rows in codec space: permutation (ProfilePerm) or rotation.
__device__ __forceinline__ void unit_codec_rows(const DecodeParams& p, const float (*qo)[128],
                                                float (*qc)[128], int tid, int nthr) {
  for (int e = tid; e < p.R * p.d; e += nthr) {
    const int r = e / p.d, j = e - r * p.d;
    float v;
    if (p.rot_k) {
      float a = 0.f;
      for (int i = 0; i < p.d; ++i) a = fmaf(qo[r][i], p.rot_k[j * p.d + i], a);
      v = a;
    } else {
      v = qo[r][p.perm ? p.perm[j] : j];
    }
    qc[r][j] = v;
  }
}

// Table kernel for permutation / identity codecs with 4- or 8-dim blocks:
// grid (block b, group of kLutUnits units); thread c holds centroid row c of
// block b in registers and writes entry (b, c) of the tables of all the
// group's units, so every CTA reads one block's centroids (k * BD floats)
// once instead of every unit reading all of them. Same arithmetic as
// lut_kernel: query rows dtype(q * scale) (attention.py:208), picked through
// the permutation, fused multiply-adds in dim order, zero for pass-through
// blocks.
constexpr int kLutUnits = 4;
// Fused cache append, one CTA per (key block b, 8 appended rows): warp w
// quantizes row 8a + w, lane l scans centroids l, l + 32, ... (up to 256) in
// order with a strict '<', and the lanes' winners are combined by (distance,
// index) -- the first index whose distance is below every earlier one, as the
// reference's sequential loop and ss_cache_append (NaN distances never win; a
// NaN distance at index 0, or no finite distance, gives index 0). Distances
// in NumPy's order (dist_direct). Heavy blocks store the fp16 key values and
// index 0. CTAs of block 0 also store the value rows.
constexpr int kAppRows = 8;
template <int BD>
__device__ __forceinline__ void append_rows(const DecodeParams& p, int b, int64_t a) {
  __shared__ float s_krow[kAppRows][129];  // the rows' keys, original basis
  __shared__ int s_col[BD];
  __shared__ __align__(16) float s_c[256 * BD];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t n_rows = (int64_t)p.b * p.hkv * p.app_rows;
  const int64_t r = a * kAppRows + warp;
  const bool valid = r < n_rows;
  int64_t pair = 0, tt = 0;
  if (valid) { pair = r / p.app_rows; tt = r - pair * p.app_rows; }
  const int64_t pos = p.tc - p.app_rows + tt;
  const bool heavy = p.n_heavy > 0 && p.heavy && p.heavy[b];
  // Codec state (the block's permutation and centroids) is staged before
  // griddepcontrol.wait, the step's inputs (key and value rows) after it, all
  // before the one barrier: the CTA waits for one memory latency after the
  // previous kernel.
  if (tid < BD) s_col[tid] = p.perm ? __ldg(p.perm + b * BD + tid) : b * BD + tid;
  constexpr int kPer = 8;  // centroids per lane (256 / 32)
  if (!heavy) {
    const float* cb = p.cents + (size_t)b * p.k * BD;
    for (int e = tid * 4; e < p.k * BD; e += 1024)
      *reinterpret_cast<float4*>(s_c + e) = __ldg(reinterpret_cast<const float4*>(cb + e));
  }
  grid_dependency_wait();  // the rows may come from, and the streams be read by, earlier kernels
  const int64_t kbase = pair * p.app_kps + tt * p.app_krs;
  for (int j = lane; j < p.d; j += 32)
    s_krow[warp][j] = valid ? load_as_f32(p.app_k, p.app_dt, kbase + j) : 0.f;
  if (b == 0 && valid) {
    // this warp's value row, as fp16, in 8-element chunks whose loads all
    // issue before their stores (source and destination may alias as far as
    // the compiler knows)
    const int64_t src0 = pair * p.app_vps + tt * p.app_vrs;
    for (int j0 = lane * 8; j0 < p.d; j0 += 256) {
      float x[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = load_as_f32(p.app_v, p.app_dt, src0 + j0 + j);
      uint4 h;
      h.x = pack_h2(x[0], x[1]); h.y = pack_h2(x[2], x[3]);
      h.z = pack_h2(x[4], x[5]); h.w = pack_h2(x[6], x[7]);
      *reinterpret_cast<uint4*>(p.v_w + pair * p.v_ps + pos * p.d + j0) = h;
    }
  }
  __syncthreads();
  if (!valid) return;
  float kk[BD];
#pragma unroll
  for (int j = 0; j < BD; ++j) kk[j] = s_krow[warp][s_col[j]];
  if (heavy) {
    if (lane == 0) {
      int hpos = 0;
      for (int bb = 0; bb < b; ++bb) hpos += p.heavy[bb] ? 1 : 0;
      uint16_t* dst = const_cast<uint16_t*>(p.kheavy) + pair * p.kh_ps +
                      pos * (p.n_heavy * p.bd) + hpos * BD;
#pragma unroll
      for (int j = 0; j < BD; ++j) dst[j] = f2h(kk[j]);
      const_cast<uint8_t*>(p.idx)[pair * p.idx_ps + pos * p.nb + b] = 0;
    }
    return;
  }
  float dd[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int c = lane + 32 * i;
    dd[i] = c < p.k ? dist_direct<BD>(kk, s_c + c * BD) : 0.f;
  }
  float best = __int_as_float(0x7f800000);
  int bi = 0x7fffffff;
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    if (lane + 32 * i < p.k && dd[i] < best) { best = dd[i]; bi = lane + 32 * i; }
  const float d0 = __shfl_sync(0xffffffffu, dd[0], 0);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob < best || (ob == best && oi < bi)) { best = ob; bi = oi; }
  }
  if (lane == 0) {
    const int idx = (d0 != d0 || bi == 0x7fffffff) ? 0 : bi;
    const_cast<uint8_t*>(p.idx)[pair * p.idx_ps + pos * p.nb + b] = static_cast<uint8_t>(idx);
  }
}

template <int R, int BD>
__global__ void __launch_bounds__(256, 4) lut_block_kernel(const __grid_constant__ DecodeParams p) {
  __shared__ __align__(16) float qs[kLutUnits][R][BD];
  const int tid = threadIdx.x;
  const int b = blockIdx.x;
  // This kernel is launched as a programmatic dependent of the kernel before
  // it (typically the previous step's decode, which signals at its start):
  // before griddepcontrol.wait it reads only codec state (centroids,
  // permutation, heavy-block mask), which no kernel that signals early writes.
  if ((int)blockIdx.y >= p.lut_groups) {  // fused cache append
    grid_launch_dependents();
    append_rows<BD>(p, b, (int64_t)blockIdx.y - p.lut_groups);  // waits inside
    return;
  }
  const int64_t u0 = (int64_t)blockIdx.y * kLutUnits;
  grid_launch_dependents();  // let the decode grid start streaming now
  const int c = tid;
  const bool zero = p.n_heavy > 0 && p.heavy && p.heavy[b];
  float cv[BD];
#pragma unroll
  for (int j = 0; j < BD; j += 4) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < p.k) v = __ldg(reinterpret_cast<const float4*>(p.cents + ((size_t)b * p.k + c) * BD + j));
    cv[j] = v.x; cv[j + 1] = v.y; cv[j + 2] = v.z; cv[j + 3] = v.w;
  }
  // Each thread's query element (at most one: kLutUnits * R * BD <= 256):
  // its offset, with the permutation column, is found before the wait (the
  // permutation is codec state), so only the query load follows it.
  static_assert(kLutUnits * R * BD <= 256, "one query element per thread");
  const int rows_valid = p.nrep * p.tq;
  const int e = tid;
  const int ui = e / (R * BD), rem = e - ui * (R * BD), r = rem / BD, j = rem - r * BD;
  int64_t qoff = -1;
  if (e < kLutUnits * R * BD && u0 + ui < p.n_units) {
    const int64_t u = u0 + ui;
    const int64_t pair = u / p.n_rg;
    const int rg = static_cast<int>(u - pair * p.n_rg);
    const int bb = static_cast<int>(pair / p.hkv), hh = static_cast<int>(pair % p.hkv);
    const int rr = rg * R + r;
    if (rr < rows_valid) {
      const int rep = rr / p.tq, tqi = rr - rep * p.tq;
      const int qh = hh * p.nrep + rep;
      const int col = p.perm ? __ldg(p.perm + b * BD + j) : b * BD + j;
      qoff = bb * p.q_sb + qh * p.q_sh + tqi * p.q_st + col;
    }
  }
  grid_dependency_wait();  // queries, and the table slots the previous decode reads
  if (e < kLutUnits * R * BD) {
    const float sc = round_to(p.scale, p.qdt);
    qs[ui][r][j] = qoff < 0 ? 0.f : round_to(load_as_f32(p.q, p.qdt, qoff) * sc, p.qdt);
  }
  __syncthreads();
  if (c >= p.k) return;
#pragma unroll 2
  for (int ui = 0; ui < kLutUnits; ++ui) {
    const int64_t u = u0 + ui;
    if (u >= p.n_units) break;
    float o[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float qv[BD];
#pragma unroll
      for (int j = 0; j < BD; j += 4) {
        const float4 q4 = *reinterpret_cast<const float4*>(&qs[ui][r][j]);
        qv[j] = q4.x; qv[j + 1] = q4.y; qv[j + 2] = q4.z; qv[j + 3] = q4.w;
      }
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < BD; ++j) acc = fmaf(zero ? 0.f : qv[j], cv[j], acc);
      o[r] = acc;
    }
    float* dst = p.lut_g + (size_t)u * (p.lut_unit_bytes / 4) + ((size_t)b * p.k + c) * R;
    if constexpr (R % 4 == 0) {
#pragma unroll
      for (int r = 0; r < R; r += 4)
        *reinterpret_cast<float4*>(dst + r) = make_float4(o[r], o[r + 1], o[r + 2], o[r + 3]);
    } else {
#pragma unroll
      for (int r = 0; r < R; ++r) dst[r] = o[r];
    }
  }
}

// Grid (units, block chunks): CTA (u, g) computes the table of blocks
// [g * kLutBlocks, (g + 1) * kLutBlocks) of unit u into the workspace, laid
// out [unit][nb][k][R]. Thread t owns block b0 + t / 64 (its R query
// sub-vectors in registers) and centroids t % 64 + i * 64, so a warp writes
// contiguous table rows.
// BD = 0 is the generic path for block sizes other than 4 and 8.
constexpr int kLutBlocks = 8;
template <int R, int BD>
__global__ void __launch_bounds__(kLutThreads) lut_kernel(const __grid_constant__ DecodeParams p) {
  // only this unit's R query rows (keeps the CTA small enough to share an SM
  // with a decode CTA)
  __shared__ float qo[R][128], qc[R][128];
  const int tid = threadIdx.x;
  const int64_t u = blockIdx.x;
  const int b0 = blockIdx.y * kLutBlocks;
  const int64_t pair = u / p.n_rg;
  const int rg = static_cast<int>(u - pair * p.n_rg);
  const int bb = static_cast<int>(pair / p.hkv), hh = static_cast<int>(pair % p.hkv);
  grid_launch_dependents();  // let the decode grid start streaming now
  float* out = p.lut_g + (size_t)u * (p.lut_unit_bytes / 4);
  if constexpr (BD > 0) {
    if (p.rot_k == nullptr) {
      // Identity / permutation codecs: every global load (centroids, the
      // block's permutation entries, the query rows) is issued up front so the
      // kernel pays one memory latency, then one barrier.
      constexpr int TPB = kLutThreads / kLutBlocks;
      const int b = b0 + tid / TPB, cl = tid % TPB;
      const bool bok = b < p.nb;
      const float* cb = p.cents + (size_t)(bok ? b : 0) * p.k * BD;
      constexpr int NCV = (256 + TPB - 1) / TPB;  // centroid rows per thread (k <= 256)
      float cv[NCV][BD];
#pragma unroll
      for (int i = 0; i < NCV; ++i) {
        const int c = cl + i * TPB;
#pragma unroll
        for (int j = 0; j < BD; j += 4) {
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (bok && c < p.k) v = __ldg(reinterpret_cast<const float4*>(cb + (size_t)c * BD + j));
          cv[i][j] = v.x; cv[i][j + 1] = v.y; cv[i][j + 2] = v.z; cv[i][j + 3] = v.w;
        }
      }
      int pj[BD];
#pragma unroll
      for (int j = 0; j < BD; ++j) {
        const int col = (bok ? b : 0) * BD + j;
        pj[j] = p.perm ? __ldg(p.perm + col) : col;
      }
      constexpr int QPT = (R * 128 + kLutThreads - 1) / kLutThreads;
      const float sc = round_to(p.scale, p.qdt);
      const int rows_valid = p.nrep * p.tq;
      float qv[QPT];
#pragma unroll
      for (int i = 0; i < QPT; ++i) {
        const int e = tid + i * kLutThreads;
        const int r = e / p.d, j = e - r * p.d;
        const int rr = rg * R + r;
        qv[i] = 0.f;
        if (e < R * p.d && rr < rows_valid) {
          const int rep = rr / p.tq, tqi = rr - rep * p.tq;
          const int qh = hh * p.nrep + rep;
          qv[i] = load_as_f32(p.q, p.qdt, bb * p.q_sb + qh * p.q_sh + tqi * p.q_st + j);
        }
      }
#pragma unroll
      for (int i = 0; i < QPT; ++i) {
        const int e = tid + i * kLutThreads;
        const int r = e / p.d, j = e - r * p.d;
        if (e < R * p.d) qo[r][j] = round_to(qv[i] * sc, p.qdt);  // attention.py:208
      }
      __syncthreads();
      if (!bok) return;
      const bool zero = p.n_heavy > 0 && p.heavy && p.heavy[b];
      float q[R][BD];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int j = 0; j < BD; ++j) q[r][j] = zero ? 0.f : qo[r][pj[j]];
      float* ob = out + (size_t)b * p.k * R;
#pragma unroll
      for (int i = 0; i < NCV; ++i) {
        const int c = cl + i * TPB;
        if (c >= p.k) break;
        float o[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float acc = 0.f;
#pragma unroll
          for (int j = 0; j < BD; ++j) acc = fmaf(q[r][j], cv[i][j], acc);
          o[r] = acc;
        }
        float* dst = ob + (size_t)c * R;
        if constexpr (R % 4 == 0) {
#pragma unroll
          for (int r = 0; r < R; r += 4)
            *reinterpret_cast<float4*>(dst + r) = make_float4(o[r], o[r + 1], o[r + 2], o[r + 3]);
        } else {
#pragma unroll
          for (int r = 0; r < R; ++r) dst[r] = o[r];
        }
      }
      return;
    }
  }
  unit_query_rows(p, qo, rg, bb, hh, tid, kLutThreads);
  __syncthreads();
  unit_codec_rows(p, qo, qc, tid, kLutThreads);
  __syncthreads();
  if constexpr (BD > 0) {
    const int b = b0 + tid / (kLutThreads / kLutBlocks);
    if (b >= p.nb) return;
    const bool zero = p.n_heavy > 0 && p.heavy && p.heavy[b];
    float q[R][BD];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int j = 0; j < BD; ++j) q[r][j] = zero ? 0.f : qc[r][b * BD + j];
    const float* cb = p.cents + (size_t)b * p.k * BD;
    float* ob = out + (size_t)b * p.k * R;
#pragma unroll 4
    for (int c = tid % (kLutThreads / kLutBlocks); c < p.k; c += kLutThreads / kLutBlocks) {
      float cv[BD];
#pragma unroll
      for (int j = 0; j < BD; j += 4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(cb + (size_t)c * BD + j));
        cv[j] = v.x; cv[j + 1] = v.y; cv[j + 2] = v.z; cv[j + 3] = v.w;
      }
      float o[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < BD; ++j) acc = fmaf(q[r][j], cv[j], acc);
        o[r] = acc;
      }
      float* dst = ob + (size_t)c * R;
      if constexpr (R % 4 == 0) {
#pragma unroll
        for (int r = 0; r < R; r += 4)
          *reinterpret_cast<float4*>(dst + r) = make_float4(o[r], o[r + 1], o[r + 2], o[r + 3]);
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) dst[r] = o[r];
      }
    }
  } else {
    const int nbl = min(kLutBlocks, p.nb - b0);
    for (int e = tid; e < nbl * p.k; e += kLutThreads) {
      const int b = b0 + e / p.k, c = e % p.k;
      const bool zero = p.n_heavy > 0 && p.heavy && p.heavy[b];
      const float* cv = p.cents + ((size_t)b * p.k + c) * p.bd;
      float* dst = out + ((size_t)b * p.k + c) * R;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float acc = 0.f;
        for (int j = 0; j < p.bd; ++j) acc = fmaf(qc[r][b * p.bd + j], __ldg(cv + j), acc);
        dst[r] = zero ? 0.f : acc;
      }
    }
  }
}

template <int R, int D, int NBC, int CW, bool HV, int LEAN = 0>
__global__ void __launch_bounds__(CW * 32 + 32, 1) decode_attn_kernel(
    const __grid_constant__ DecodeParams p, const __grid_constant__ CUtensorMap map_v,
    const __grid_constant__ CUtensorMap map_vt) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Align to 1024 B (128-byte-swizzle atoms) by an offset from the __shared__
  // array itself, so every access below stays a shared-memory access.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint64_t full_bar[kMaxStages], empty_bar[kMaxStages], lut_bar;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  constexpr int TILE = 128;
  Misc& ms = *reinterpret_cast<Misc*>(smem + p.off_misc);
  float* lut = reinterpret_cast<float*>(smem + p.off_lut);

  // The next step's table kernel may launch now: it waits for this grid
  // before it reads or writes anything this grid uses.
  grid_launch_dependents();
  const int64_t cta = blockIdx.x;
  const Sched sched = make_sched(p.total_tiles, p.tpu, p.w_unit, p.grid);
  const int64_t t_begin = range_start(sched, cta);
  const int64_t t_end = range_start(sched, cta + 1);

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], TILE / slice_tokens(R));
    }
    mbar_init(&lut_bar, 1);
    ms.abort = 0;
    int hp = 0;
    for (int b = 0; b < p.nb; ++b) {
      const bool hv = p.heavy && p.heavy[b];
      ms.is_heavy[b] = hv ? 1 : 0;
      if (hv && hp < 32) ms.heavy_pos[hp++] = b;
    }
    for (int i = 0; i < 16; ++i) ms.levels[i] = p.levels[i];
    for (int i = 0; i < 16; ++i) ms.lvpair[i] = make_float2(p.levels[i & 3], p.levels[i >> 2]);

    fence_mbar_init();
  }
  __syncthreads();

  // ====================================================== producer warp
  if (warp == CW) {
    if (lane == 0) {
      if (p.vfmt == SS_V_F16 && p.n_ct > 0) prefetch_tmap(&map_v);
      if (p.n_tt > 0 && p.vfmt == SS_V_F16) prefetch_tmap(&map_vt);
      int it = 0;
      // walk (unit, tile) incrementally: no per-tile 64-bit division
      int64_t u = t_begin / p.tpu;
      int lt = static_cast<int>(t_begin - u * p.tpu);
      int64_t pair = u / p.n_rg;
      int rgc = static_cast<int>(u - pair * p.n_rg);
      int s = 0, ph = 0;  // stage of tile `it` and its use count parity
      bool dep_done = false;
      for (int64_t tau = t_begin; tau < t_end; ++tau, ++it) {
        if (tau != t_begin && ++lt == p.tpu) {
          lt = 0;
          ++u;
          if (++rgc == p.n_rg) { rgc = 0; ++pair; }
        }
        if (it > 0 && ++s == p.stages) { s = 0; ph ^= 1; }
        if (it >= p.stages) {
          if (ms.abort || !mbar_wait_bounded(&empty_bar[s], ph ^ 1, p.wait_ns)) {
            if (!ms.abort) report_wait_failure(p.err, p.sink, 1);
            ms.abort = 1;
            break;
          }
        }
        uint8_t* st = smem + (size_t)s * p.stage_bytes;
        if (lt < p.n_ct) {
          const int64_t t0 = (int64_t)lt * TILE;
          // tokens appended by this step's table kernel (the primary of this
          // programmatic dependent launch): wait for it before reading them
          if (p.app_rows > 0 && !dep_done && t0 + TILE > p.tc - p.app_rows) {
            grid_dependency_wait();
            dep_done = true;
          }
          uint32_t bytes = TILE * p.nb;
          if (p.vfmt == SS_V_F16) bytes += TILE * D * 2;
          else bytes += p.v_tile_bytes;
          if (p.n_heavy) bytes += TILE * p.n_heavy * p.bd * 2;
          mbar_arrive_expect_tx(&full_bar[s], bytes);
          if (tau == p.skip_tile) continue;  // test hook: these bytes never arrive
          bulk_g2s(st + p.off_idx, p.idx + pair * p.idx_ps + t0 * p.nb, TILE * p.nb,
                   &full_bar[s]);
          uint8_t* aux = st + p.off_aux;
          if (p.vfmt == SS_V_F16) {
            for (int bx = 0; bx < D / 64; ++bx)
              tma_load_3d(st + bx * TILE * 128, &map_v, bx * 64, static_cast<int32_t>(t0),
                          static_cast<int32_t>(pair), &full_bar[s]);
          } else if (p.vfmt == SS_V_VQ) {
            bulk_g2s(aux, p.vidx + pair * p.vi_ps + t0 * p.v_nb, TILE * p.v_nb, &full_bar[s]);
            aux += TILE * p.v_nb;
          } else {
            const uint32_t wb = TILE * p.v_words * 4;
            bulk_g2s(aux, p.vq + pair * p.vq_ps + t0 * p.v_words, wb, &full_bar[s]);
            aux += wb;
            const int sb = p.vs_dt == SS_F32 ? 4 : 2;
            const uint32_t sbytes = TILE * p.v_groups * sb;
            bulk_g2s(aux, reinterpret_cast<const uint8_t*>(p.vs) +
                              (pair * p.vs_ps + t0 * p.v_groups) * sb,
                     sbytes, &full_bar[s]);
            aux += sbytes;
            if (p.vz) {
              bulk_g2s(aux, p.vz + pair * p.vz_ps + t0 * p.v_groups, TILE * p.v_groups * 4,
                       &full_bar[s]);
              aux += TILE * p.v_groups * 4;
            }
          }
          if (p.n_heavy) {
            const uint32_t hb = TILE * p.n_heavy * p.bd * 2;
            bulk_g2s(aux, p.kheavy + pair * p.kh_ps + t0 * p.n_heavy * p.bd, hb, &full_bar[s]);
          }
        } else {
          const int64_t t0 = (int64_t)(lt - p.n_ct) * TILE;
          if (p.vfmt == SS_V_F16) {
            mbar_arrive_expect_tx(&full_bar[s], TILE * D * 2);
            for (int bx = 0; bx < D / 64; ++bx)
              tma_load_3d(st + bx * TILE * 128, &map_vt, bx * 64, static_cast<int32_t>(t0),
                          static_cast<int32_t>(pair), &full_bar[s]);
          } else {
            mbar_arrive(&full_bar[s]);  // consumers read the tail directly
          }
        }
      }
      // Drain: make sure no copy issued by this CTA is still in flight. Each
      // stage is waited for separately (a stage whose bytes never arrive
      // must not stop the wait for the others).
      const int issued = it;
      bool drained = true;
      for (int j = issued - p.stages; j < issued; ++j) {
        if (j < 0) continue;
        const int s = j % p.stages;
        if (!mbar_wait_bounded(&full_bar[s], (j / p.stages) & 1, p.wait_ns)) drained = false;
      }
      if (!drained) report_wait_failure(p.err, p.sink, 2);
    }
    return;
  }

  // ====================================================== consumer warps
  // Warp w owns 64-token slice (w % wps) of every tile of its tile group
  // (w / wps); lane l scores tokens l and l + 32 of the slice over all blocks.
  constexpr int MT = D / 16;                   // 16-dim MMA tiles of the output
  constexpr int TPL = slice_tokens(R) / 32;    // tokens per lane
  constexpr int SL = 32 * TPL;                 // tokens per warp slice
  const int wps = TILE / SL;                   // warps sharing one tile
  const int tgroups = CW / wps;
  const int wgroup = warp / wps, slice = warp % wps;
  const int ctid = tid;                        // 0..255
  const int64_t q_off = p.tc + p.ttail - p.tq;
  // Softmax weights go to the P.V MMA as fp16 hi + lo pairs (p = hi + lo to
  // about 2^-22 relative), so the weighted sum has fp32-level accuracy. With
  // R <= 4 rows the lo halves sit in columns 4..7 of the same 8-column slice
  // (one MMA computes both; the two column halves are added at the unit
  // end); with 8 rows they have a slice of their own and a second MMA.
  __half* Pw = reinterpret_cast<__half*>(smem + p.off_p) + warp * SL * 8;  // [32][8]
  __half* Pw_lo = R == 8 ? reinterpret_cast<__half*>(p.off_plo ? smem + p.off_plo
                                                               : reinterpret_cast<uint8_t*>(&ms.qo[0][0])) +
                               warp * SL * 8
                         : Pw;
  uint8_t* vdq_w = smem + p.off_vdq + warp * (16 * D * 2);
  const uint32_t pw_addr = smem_u32(Pw) + (lane & 15) * 16;
  const uint32_t pwl_addr = smem_u32(Pw_lo) + (lane & 15) * 16;
  // ldmatrix.x4.trans addressing: lane -> (8x8 matrix mi, row mj)
  const int mi = lane >> 3, mj = lane & 7;
  const int kk_off = (mi >= 2 ? 8 : 0) + mj;   // token row within a 16-token k-step
  const int dsel = mi & 1;                     // second 8-dim half of the 16-dim tile
  // 128-byte-swizzle chunk offset of 16-dim MMA tile m (and m + 4 in the next box)
  uint32_t swz[4];
#pragma unroll
  for (int m = 0; m < 4; ++m) swz[m] = static_cast<uint32_t>(((2 * m + dsel) ^ mj) << 4);
  const int rows_valid = p.nrep * p.tq;
  const bool per_token_mask = LEAN ? false : (p.causal || p.mask != nullptr);
  const int vdec = (LEAN == 1 || LEAN == 3) ? 0 : LEAN == 2 ? 4 : LEAN == 4 ? 2 : p.vdec;
  // LEAN 2: the four levels of the 2-bit codes split into fp16 heads and
  // fp16 remainders (level = head + remainder to ~2^-22), as byte-permute
  // sources: low bytes of levels 0..3 in *_lo, high bytes in *_hi
  uint32_t lv_lo = 0, lv_hi = 0, lw_lo = 0, lw_hi = 0;
  if constexpr (LEAN == 2) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const __half hh = __float2half_rn(p.levels[c]);
      const uint32_t h = __half_as_ushort(hh);
      const uint32_t l = __half_as_ushort(__float2half_rn(p.levels[c] - __half2float(hh)));
      lv_lo |= (h & 0xffu) << (8 * c);
      lv_hi |= (h >> 8) << (8 * c);
      lw_lo |= (l & 0xffu) << (8 * c);
      lw_hi |= (l >> 8) << (8 * c);
    }
  }
  // vdec 4: this lane's byte offsets (from the stage base, first 16-token
  // step) of its four packed value words and of its two fp16 group scales
  const uint32_t q4_word_off =
      p.off_aux + (uint32_t)(((warp % (TILE / SL)) * SL + (lane >> 1)) * 8 + (lane & 1) * 4) * 4;
  const uint32_t q4_scale_off = p.off_aux + TILE * 8 * 4 +
      (uint32_t)(((warp % (TILE / SL)) * SL + (lane >> 1)) * 4 + (lane & 1) * 2) * 2;
  // columns of every P slice that no row uses stay zero
  if constexpr (R < 4) {
    for (int e = lane; e < SL * 8; e += 32)
      if ((e & 3) >= R) Pw[e] = __float2half_rn(0.f);
  }

  // Heavy (fp16 pass-through) blocks score on warp MMAs when their dims fit
  // 16-dim k-steps: A = 16 tokens x 16 heavy dims straight from the stage,
  // B = the unit's heavy query rows split into fp16 hi + lo (fp32-level
  // accuracy); the 16x8 fp32 results go back to one token per lane through
  // the warp's P slice, which is free between P.V and the next softmax.
  const int hd = p.n_heavy * p.bd;
  const uint32_t heavy_off = p.off_aux + (p.vfmt == SS_V_F16 ? 0u : p.v_tile_bytes);
  const bool heavy_mma_shape = HV && (R == 4 || R == 8) && SL == 32 && p.n_heavy > 0 &&
                               hd % 16 == 0 && hd <= 64 && (heavy_off & 15u) == 0;
  // B fragments [k-step][hi, lo][lane] (b0, b1), kept in the codec-query rows
  // once those are built into fragments (nothing else reads them then)
  const uint2* hqs = reinterpret_cast<const uint2*>(&ms.qc[0][0]);
  bool heavy_mma = false;

  if ((!LEAN || LEAN == 4) && p.vfmt == SS_V_VQ) {
    // value centroids, once per CTA: [v_nb][256][v_bd] fp16 with entries
    // c >= v_k zeroed, so any stored index byte reads a finite row (the
    // unit loop's first barrier publishes the table)
    uint16_t* vt = reinterpret_cast<uint16_t*>(smem + p.off_vtab);
    for (int cid = ctid; cid < p.v_nb * 256; cid += CW * 32) {
      const int b = cid >> 8, c = cid & 255;
      const bool ok = c < p.v_k;
      const uint16_t* src = p.vcents + ((size_t)b * p.v_k + c) * p.v_bd;
      uint16_t* dst = vt + (size_t)cid * p.v_bd;
      if (p.v_bd == 4) {
        *reinterpret_cast<uint2*>(dst) = ok ? __ldg(reinterpret_cast<const uint2*>(src)) : make_uint2(0, 0);
      } else {
        for (int j = 0; j < p.v_bd; j += 8)
          *reinterpret_cast<uint4*>(dst + j) =
              ok ? __ldg(reinterpret_cast<const uint4*>(src + j)) : make_uint4(0, 0, 0, 0);
      }
    }
  }

  int64_t tau = t_begin;
  uint32_t unit_no = 0;
  bool lut_out = false;     // thread 0: a table copy whose completion was not seen
  uint32_t lut_phase = 0;
  while (tau < t_end) {
    const int64_t u = tau / p.tpu;
    const int64_t u_end = min(t_end, (u + 1) * p.tpu);
    const int64_t pair = u / p.n_rg;
    const int rg = static_cast<int>(u - pair * p.n_rg);
    const int bb = static_cast<int>(pair / p.hkv), hh = static_cast<int>(pair % p.hkv);

    // ---------------------------------------------- the unit's LUT
    // Tables are precomputed for all units by lut_kernel; one bulk copy brings
    // this unit's table into shared memory. Query rows are only needed here
    // for exact dot products (fp16 tail tokens, heavy blocks).
    named_bar_sync(1, (CW * 32));  // previous unit finalised, LUT region free
    if (ctid == 0) {
      // Tables come from lut_kernel, launched just before as the primary of a
      // programmatic dependent launch: wait for its results once.
      if (unit_no == 0) grid_dependency_wait();
    }
    // after a give-up no further table copy is issued (so at most one, whose
    // wait was skipped, can still be in flight: drained at the end)
    if (ctid == 0 && !ms.abort) {
      lut_out = true;
      lut_phase = unit_no & 1;
      fence_proxy_async_smem();  // region was last written as merge scratch
      const uint32_t bytes = p.lut_unit_bytes;
      mbar_arrive_expect_tx(&lut_bar, bytes);
      const uint8_t* src = reinterpret_cast<const uint8_t*>(p.lut_g) + (size_t)u * bytes;
      for (uint32_t off = 0; off < bytes; off += 16384u)
        bulk_g2s(reinterpret_cast<uint8_t*>(lut) + off, src + off,
                 bytes - off < 16384u ? bytes - off : 16384u, &lut_bar);
    }
    if ((!LEAN || LEAN == 3) && (p.ttail > 0 || p.n_heavy > 0)) {
      unit_query_rows(p, ms.qo, rg, bb, hh, ctid, (CW * 32));
      named_bar_sync(1, (CW * 32));
      unit_codec_rows(p, ms.qo, ms.qc, ctid, (CW * 32));
      named_bar_sync(1, (CW * 32));
      if (heavy_mma_shape) {
        // B fragment of m16n8k16: b0 = B[2t, 2t+1][g], b1 = B[2t+8, 2t+9][g]
        // with B[e][n] = codec-space query row n at heavy dim e.
        const int g = lane >> 2, t = lane & 3;
        bool finite = true;
        uint32_t hq[4][2][2];  // [k-step][hi, lo][b0, b1]
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          if (ks * 16 >= hd) break;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float qv[2];
            __half hi[2], lo[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int e = ks * 16 + h * 8 + 2 * t + j;
              const int hb = e / p.bd;
              qv[j] = g < R ? ms.qc[g][ms.heavy_pos[hb] * p.bd + (e - hb * p.bd)] : 0.f;
              hi[j] = __float2half_rn(qv[j]);
              lo[j] = __float2half_rn(qv[j] - __half2float(hi[j]));
              finite = finite && isfinite(__half2float(hi[j])) && isfinite(__half2float(lo[j]));
            }
            hq[ks][0][h] = pack_halves2(hi[0], hi[1]);
            hq[ks][1][h] = pack_halves2(lo[0], lo[1]);
          }
        }
        heavy_mma = __all_sync(0xffffffffu, finite);
        named_bar_sync(1, (CW * 32));  // every warp has read the codec rows
        if (heavy_mma && warp == 0) {
          uint2* dst = reinterpret_cast<uint2*>(&ms.qc[0][0]);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            if (ks * 16 >= hd) break;
            dst[(ks * 2 + 0) * 32 + lane] = make_uint2(hq[ks][0][0], hq[ks][0][1]);
            dst[(ks * 2 + 1) * 32 + lane] = make_uint2(hq[ks][1][0], hq[ks][1][1]);
          }
        }
        named_bar_sync(1, (CW * 32));
      }
    }
    if (!ms.abort) {
      if (mbar_wait_bounded(&lut_bar, unit_no & 1, p.wait_ns)) {
        lut_out = false;
      } else {
        ms.abort = 1;
        report_wait_failure(p.err, p.sink, 8);
      }
    }
    ++unit_no;
    uint32_t rok = 0;  // bit r: query row r of this unit exists
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (rg * R + r < rows_valid) rok |= 1u << r;

    // ---------------------------------------------- this warp's slices of the unit
    float m_w[R], l_l[R];
    float acc[MT][4];
#pragma unroll
    for (int r = 0; r < R; ++r) { m_w[r] = -INFINITY; l_l[r] = 0.f; }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;

    // this warp's tiles of the unit: it = tau - t_begin + i with it % tgroups == wgroup
    const int it0 = static_cast<int>(tau - t_begin);
    const int lt0 = static_cast<int>(tau - u * p.tpu);
    const int n_here = static_cast<int>(u_end - tau);
    const int ifirst = (wgroup - it0 % tgroups + tgroups) % tgroups;
    // stage and phase of this warp's first tile; later tiles advance by the
    // number of tile groups, which divides the stage count
    int s = (it0 + ifirst) % p.stages, ph = ((it0 + ifirst) / p.stages) & 1;
    for (int i = ifirst; i < n_here; i += tgroups) {
      if (i != ifirst) {
        s += tgroups;
        if (s >= p.stages) { s -= p.stages; ph ^= 1; }
      }
      const int lt = lt0 + i;
      if (!ms.abort && !mbar_wait_bounded(&full_bar[s], ph, p.wait_ns)) {
        ms.abort = 1;
        report_wait_failure(p.err, p.sink, 4);
      }
      const bool aborted = ms.abort != 0;
      uint8_t* st = smem + (size_t)s * p.stage_bytes;
      const bool compressed = LEAN ? true : lt < p.n_ct;
      const int t0 = (compressed ? lt : lt - p.n_ct) * TILE;
      const int rem_ = static_cast<int>(compressed ? p.tc : p.ttail) - t0;
      const int len = rem_ < TILE ? rem_ : TILE;
      const int tok0 = slice * SL + lane;       // tokens of this lane within the tile
      const int tok1 = TPL > 1 ? tok0 + 32 : tok0;
      const bool v0 = tok0 < len && !aborted, v1 = TPL > 1 && tok1 < len && !aborted;

      // 1. scores
      float s0[R], s1[R];
#pragma unroll
      for (int r = 0; r < R; ++r) { s0[r] = 0.f; s1[r] = 0.f; }
      if (compressed) {
        const uint8_t* ir0 = st + p.off_idx + tok0 * p.nb;
        const uint8_t* ir1 = st + p.off_idx + tok1 * p.nb;
        if constexpr (NBC > 0 && R % 4 == 0 && TPL == 1) {
          // 16 blocks: each (block, centroid) row of the table is R floats;
          // R/2 packed fp32 pair accumulators take the 16-byte loads as two
          // 64-bit halves (no register shuffling between the load and the
          // packed add); block order as in the generic loop below
          uint64_t acc2[R / 2];
#pragma unroll
          for (int i = 0; i < R / 2; ++i) acc2[i] = 0ull;
          const uint32_t lbase = smem_u32(lut);
          // the token's index bytes in one 16-byte load per 16 blocks (lanes
          // read consecutive 16-byte rows: no bank conflicts)
          uint32_t cw4[NBC / 4];
#pragma unroll
          for (int w = 0; w < NBC / 4; w += 4) {
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (v0) v = *reinterpret_cast<const uint4*>(ir0 + 4 * w);
            cw4[w] = v.x; cw4[w + 1] = v.y; cw4[w + 2] = v.z; cw4[w + 3] = v.w;
          }
#pragma unroll
          for (int w = 0; w < NBC / 4; ++w) {
            const uint32_t c0w = cw4[w];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t a = lbase + ((4 * w + j) * 256u * R + __byte_perm(c0w, 0u, 0x4440u + j) * R) * 4u;
#pragma unroll
              for (int r4 = 0; r4 < R; r4 += 4) {
                uint64_t x, y;
                asm("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "r"(a + r4 * 4));
                asm("add.rn.f32x2 %0, %0, %1;" : "+l"(acc2[r4 / 2]) : "l"(x));
                asm("add.rn.f32x2 %0, %0, %1;" : "+l"(acc2[r4 / 2 + 1]) : "l"(y));
              }
            }
          }
#pragma unroll
          for (int i = 0; i < R / 2; ++i)
            asm("mov.b64 {%0, %1}, %2;" : "=f"(s0[2 * i]), "=f"(s0[2 * i + 1]) : "l"(acc2[i]));
        } else if (NBC > 0 || (p.nb & 3) == 0) {
          const int nbw = NBC > 0 ? NBC / 4 : (p.nb >> 2);
          // floats per block of the table (compile-time for 16 blocks x 256 centroids)
          const uint32_t kstride = NBC > 0 ? 256u * R : static_cast<uint32_t>(p.k) * R;
#pragma unroll
          for (int w = 0; w < (NBC > 0 ? NBC / 4 : 32); ++w) {
            if (NBC == 0 && w >= nbw) break;
            const uint32_t c0w = v0 ? reinterpret_cast<const uint32_t*>(ir0)[w] : 0u;
            const uint32_t c1w = v1 ? reinterpret_cast<const uint32_t*>(ir1)[w] : 0u;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t bo = (4 * w + j) * kstride;
              const float* e0 = lut + bo + __byte_perm(c0w, 0u, 0x4440u + j) * R;
              const float* e1 = lut + bo + __byte_perm(c1w, 0u, 0x4440u + j) * R;
              if constexpr (R % 4 == 0) {
#pragma unroll
                for (int r4 = 0; r4 < R; r4 += 4) {
                  const float4 a4 = *reinterpret_cast<const float4*>(e0 + r4);
                  add_f32x2(s0[r4], s0[r4 + 1], a4.x, a4.y);
                  add_f32x2(s0[r4 + 2], s0[r4 + 3], a4.z, a4.w);
                  if (TPL > 1) {
                    const float4 b4 = *reinterpret_cast<const float4*>(e1 + r4);
                    add_f32x2(s1[r4], s1[r4 + 1], b4.x, b4.y);
                    add_f32x2(s1[r4 + 2], s1[r4 + 3], b4.z, b4.w);
                  }
                }
              } else {
#pragma unroll
                for (int r = 0; r < R; ++r) {
                  s0[r] += e0[r];
                  if (TPL > 1) s1[r] += e1[r];
                }
              }
            }
          }
        } else {
          for (int b = 0; b < p.nb; ++b) {
            const float* e0 = lut + ((size_t)b * p.k + (v0 ? ir0[b] : 0)) * R;
            const float* e1 = lut + ((size_t)b * p.k + (v1 ? ir1[b] : 0)) * R;
#pragma unroll
            for (int r = 0; r < R; ++r) { s0[r] += e0[r]; s1[r] += e1[r]; }
          }
        }
        if (heavy_mma) {
          // lane -> ldmatrix row: token (lane & 15) of the 16-token tile,
          // heavy dims +8 for lanes 16..31 (matrices a0..a3 of m16n8k16)
          const uint32_t ha = smem_u32(st + heavy_off) +
                              (uint32_t)((slice * SL + (lane & 15)) * hd * 2 + (lane >> 4) * 16);
          const int g = lane >> 2, t = lane & 3;
          float* scr = reinterpret_cast<float*>(Pw);  // [32 tokens][4 rows] fp32
          float c[2][4] = {};
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            if (ks * 16 >= hd) break;
            const uint2 bh = hqs[(ks * 2 + 0) * 32 + lane], bl = hqs[(ks * 2 + 1) * 32 + lane];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
              uint32_t a0, a1, a2, a3;
              ldsm_x4(ha + (uint32_t)(mt * 16 * hd * 2 + ks * 32), a0, a1, a2, a3);
              mma_16816(c[mt], a0, a1, a2, a3, bl.x, bl.y);
              mma_16816(c[mt], a0, a1, a2, a3, bh.x, bh.y);
            }
          }
#pragma unroll
          for (int half = 0; half < R / 4; ++half) {
            __syncwarp();  // previous readers of the P slice are done
            if ((t >> 1) == half) {
              const int cc = (2 * t) & 3;
#pragma unroll
              for (int mt = 0; mt < 2; ++mt) {
                *reinterpret_cast<float2*>(scr + (mt * 16 + g) * 4 + cc) = make_float2(c[mt][0], c[mt][1]);
                *reinterpret_cast<float2*>(scr + (mt * 16 + g + 8) * 4 + cc) = make_float2(c[mt][2], c[mt][3]);
              }
            }
            __syncwarp();
            const float4 hv = *reinterpret_cast<const float4*>(scr + lane * 4);
            s0[half * 4 + 0] += hv.x;
            s0[half * 4 + 1] += hv.y;
            s0[half * 4 + 2] += hv.z;
            s0[half * 4 + 3] += hv.w;
          }
          __syncwarp();  // scratch reads done before the P store
        } else if ((!LEAN || LEAN == 3) && p.n_heavy) {
          const uint16_t* h0 = reinterpret_cast<const uint16_t*>(st + heavy_off) + (size_t)tok0 * p.n_heavy * p.bd;
          const uint16_t* h1 = reinterpret_cast<const uint16_t*>(st + heavy_off) + (size_t)tok1 * p.n_heavy * p.bd;
          for (int hj = 0; hj < p.n_heavy; ++hj) {
            const int b = ms.heavy_pos[hj];
            for (int j = 0; j < p.bd; ++j) {
              const float k0 = h2f(h0[hj * p.bd + j]), k1 = h2f(h1[hj * p.bd + j]);
#pragma unroll
              for (int r = 0; r < R; ++r) {
                const float qv = ms.qc[r][b * p.bd + j];
                s0[r] = fmaf(qv, k0, s0[r]);
                s1[r] = fmaf(qv, k1, s1[r]);
              }
            }
          }
        }
      } else {
        const uint16_t* kr0 = p.k_tail + pair * p.tail_ps + (t0 + tok0) * D;
        const uint16_t* kr1 = p.k_tail + pair * p.tail_ps + (t0 + tok1) * D;
        for (int j0 = 0; j0 < D; j0 += 8) {
          const uint4 a0 = v0 ? *reinterpret_cast<const uint4*>(kr0 + j0) : make_uint4(0, 0, 0, 0);
          const uint4 a1 = v1 ? *reinterpret_cast<const uint4*>(kr1 + j0) : make_uint4(0, 0, 0, 0);
          const uint16_t* x0 = reinterpret_cast<const uint16_t*>(&a0);
          const uint16_t* x1 = reinterpret_cast<const uint16_t*>(&a1);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float k0 = h2f(x0[j]), k1 = h2f(x1[j]);
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const float qv = ms.qo[r][j0 + j];
              s0[r] = fmaf(qv, k0, s0[r]);
              s1[r] = fmaf(qv, k1, s1[r]);
            }
          }
        }
      }
      // masking: tokens past the end -> -inf; with causal or array masks also
      // rows past the unit's last query row and the masks themselves (without
      // them a missing row only gets scores nothing reads)
      if (!per_token_mask) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          if (!v0) s0[r] = -INFINITY;
          if (!v1) s1[r] = -INFINITY;
        }
      } else {
        const int tg0 = (compressed ? t0 : static_cast<int>(p.tc) + t0) + tok0;
        const int tg1 = tg0 + 32;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const bool rv = (rok >> r) & 1u;
          bool ok0 = v0 && rv, ok1 = v1 && rv;
          const int tqr = (rg * R + r) % p.tq;
          if (p.causal) {
            ok0 = ok0 && tg0 <= q_off + tqr;
            ok1 = ok1 && tg1 <= q_off + tqr;
          }
          if (p.mask) {
            const float* mrow = p.mask + tqr * p.mask_stride;
            if (ok0) {
              const float mv = mrow[tg0];
              if (p.mask_mode == 0) s0[r] += mv; else if (mv == 0.f) s0[r] = -FLT_MAX;
            }
            if (ok1) {
              const float mv = mrow[tg1];
              if (p.mask_mode == 0) s1[r] += mv; else if (mv == 0.f) s1[r] = -FLT_MAX;
            }
          }
          if (!ok0) s0[r] = -INFINITY;
          if (!ok1) s1[r] = -INFINITY;
        }
      }

      // 2. online softmax over this warp's slice
      float alpha[R];
      __half ph0[R], pl0[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float mx = warp_max_f32(TPL > 1 ? fmaxf(s0[r], s1[r]) : s0[r]);
        const float mn = fmaxf(m_w[r], mx);
        float p0 = 0.f;
        if (mn == -INFINITY) {
          alpha[r] = 1.f;
        } else {
          const float mnl = mn * kLog2e;
          // exactly 1 when the running maximum did not move (no rescale then)
          alpha[r] = m_w[r] == mn ? 1.f : fast_exp2(fmaf(m_w[r], kLog2e, -mnl));
          p0 = fast_exp2(fmaf(s0[r], kLog2e, -mnl));
        }
        const __half h0 = __float2half_rn(p0);
        ph0[r] = h0;
        pl0[r] = __float2half_rn(p0 - __half2float(h0));
        l_l[r] = l_l[r] * alpha[r] + p0;
        m_w[r] = mn;
      }
      // this lane's weights (hi and lo halves) for all rows
      static_assert(TPL == 1, "one token per lane");
      if constexpr (R == 4) {
        *reinterpret_cast<uint4*>(Pw + lane * 8) =
            make_uint4(pack_halves2(ph0[0], ph0[1]), pack_halves2(ph0[2], ph0[3]),
                       pack_halves2(pl0[0], pl0[1]), pack_halves2(pl0[2], pl0[3]));
      } else if constexpr (R == 8) {
        *reinterpret_cast<uint4*>(Pw + lane * 8) =
            make_uint4(pack_halves2(ph0[0], ph0[1]), pack_halves2(ph0[2], ph0[3]),
                       pack_halves2(ph0[4], ph0[5]), pack_halves2(ph0[6], ph0[7]));
        *reinterpret_cast<uint4*>(Pw_lo + lane * 8) =
            make_uint4(pack_halves2(pl0[0], pl0[1]), pack_halves2(pl0[2], pl0[3]),
                       pack_halves2(pl0[4], pl0[5]), pack_halves2(pl0[6], pl0[7]));
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          Pw[lane * 8 + r] = ph0[r];
          Pw[lane * 8 + 4 + r] = pl0[r];
        }
      }
      // The running maxima rarely move after the first tiles: rescale the
      // accumulators only when one did (alpha is uniform across the warp).
      bool moved = false;
#pragma unroll
      for (int r = 0; r < R; ++r) moved = moved || alpha[r] != 1.f;
      if (moved) {
        // column n holds row n (and, for R <= 4, row n - 4's lo half)
        const int n0 = R == 8 ? 2 * (lane & 3) : (2 * (lane & 3)) & 3;
        float a0 = 1.f, a1 = 1.f;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          if (r == n0) a0 = alpha[r];
          if (r == n0 + 1) a1 = alpha[r];
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          acc[mt][0] *= a0; acc[mt][1] *= a1; acc[mt][2] *= a0; acc[mt][3] *= a1;
        }
      }
      __syncwarp();

      // 3. P.V: O^T[dims][rows] += V^T[dims][64 tokens] . P[64 tokens][rows]
      if (vdec == 0) {
        const uint32_t vb = smem_u32(st) + (slice * SL + kk_off) * 128;
#pragma unroll
        for (int ks = 0; ks < SL / 16; ++ks) {
          uint32_t b0, b1, c0 = 0, c1 = 0;
          ldsm_x2_trans(pw_addr + ks * 256, b0, b1);
          if constexpr (R == 8) ldsm_x2_trans(pwl_addr + ks * 256, c0, c1);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const uint32_t col = (mt >> 2) * (TILE * 128) + swz[mt & 3];
            uint32_t x0, x1, x2, x3;
            ldsm_x4_trans(vb + ks * 2048 + col, x0, x1, x2, x3);
            if constexpr (R == 8) mma_16816(acc[mt], x0, x1, x2, x3, c0, c1);
            mma_16816(acc[mt], x0, x1, x2, x3, b0, b1);
          }
        }
      } else if constexpr (LEAN == 2) {
        // 2-bit codes with fp16 scales per 32 channels, decoded straight into
        // the MMA's A fragments (no staging tile, no level-table loads).
        // Fragment register (dim d, tokens k, k + 1) of lane (g, t): dims
        // 16 mt + g and 16 mt + g + 8 are codes g and g + 8 of packed word mt
        // of a token; one byte permute takes the bytes holding them from the
        // two tokens' words, a shift and mask isolate the four codes, one
        // multiply-add turns them into two byte-permute selectors that pick
        // fp16 levels (low bytes in lv_lo, high bytes in lv_hi), and an fp16x2
        // multiply applies the two tokens' group scales.
        // MMA k slot kappa of a 16-token step holds token pi(kappa) =
        // (kappa & 8) + ((kappa & 7) >> 1) + 4 (kappa & 1), for A and B alike
        // (a sum over tokens does not depend on their order): lane t's four
        // tokens are then t, t + 4, t + 8, t + 12, so the four lanes that load
        // one token slot read four consecutive tokens (distinct banks).
        const int g = lane >> 2, t = lane & 3;
        const uint32_t zsel = (uint32_t)(g >> 2) * 0x1111u + 0x6240u;
        const int kap = lane & 15;
        const uint32_t pw_perm = smem_u32(Pw) + (uint32_t)((kap & 8) + ((kap & 7) >> 1) + 4 * (kap & 1)) * 16u;
        const uint32_t pwl_perm = smem_u32(Pw_lo) + (uint32_t)((kap & 8) + ((kap & 7) >> 1) + 4 * (kap & 1)) * 16u;
        const uint32_t csh = 2u * (uint32_t)(g & 3);
        const uint32_t sbase = smem_u32(st) + p.off_aux;
#pragma unroll
        for (int ks = 0; ks < SL / 16; ++ks) {
          const int tok = slice * SL + ks * 16 + t;  // tokens tok, tok+4, tok+8, tok+12
          uint32_t sc2[2][4];  // [token pair][group]: (scale of the first, of the second)
#pragma unroll
          for (int pr = 0; pr < 2; ++pr) {
            uint32_t a0, a1, b0_, b1_;
            const uint32_t sa = sbase + TILE * 32 + (uint32_t)(tok + 8 * pr) * 8u;
            asm("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(a0), "=r"(a1) : "r"(sa));
            asm("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(b0_), "=r"(b1_) : "r"(sa + 32u));
            // tokens past the end (relative to the tile): zero scale, so
            // whatever their stage bytes hold, they contribute exactly 0
            // (their weights are 0 too)
            if (tok + 8 * pr >= len) a0 = a1 = 0u;
            if (tok + 8 * pr + 4 >= len) b0_ = b1_ = 0u;
            sc2[pr][0] = __byte_perm(a0, b0_, 0x5410);
            sc2[pr][1] = __byte_perm(a0, b0_, 0x7632);
            sc2[pr][2] = __byte_perm(a1, b1_, 0x5410);
            sc2[pr][3] = __byte_perm(a1, b1_, 0x7632);
          }
          uint32_t bp0, bp1, cp0 = 0, cp1 = 0;
          ldsm_x2_trans(pw_perm + ks * 256, bp0, bp1);
          if constexpr (R == 8) ldsm_x2_trans(pwl_perm + ks * 256, cp0, cp1);
#pragma unroll
          for (int qg = 0; qg < 4; ++qg) {  // scale group qg: m-tiles 2 qg, 2 qg + 1
            uint32_t w[2][2][2];  // [token pair][first, second token][word]
#pragma unroll
            for (int pr = 0; pr < 2; ++pr)
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const uint32_t wa = sbase + (uint32_t)(tok + 8 * pr + 4 * e) * 32u + qg * 8u;
                asm("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(w[pr][e][0]), "=r"(w[pr][e][1]) : "r"(wa));
              }
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const int mt = 2 * qg + i;
              uint32_t fr[2][2];  // [token pair][dim g, dim g + 8]
#pragma unroll
              for (int pr = 0; pr < 2; ++pr) {
                const uint32_t z = __byte_perm(w[pr][0][i], w[pr][1][i], zsel);
                const uint32_t c4 = (z >> csh) & 0x03030303u;
                const uint32_t sel = c4 * 0x11u + 0x40404040u;
                const uint32_t sc = sc2[pr][qg];
#pragma unroll
                for (int d8 = 0; d8 < 2; ++d8) {
                  const uint32_t sl = d8 ? sel >> 16 : sel;
                  // level = h + l (fp16 head and remainder): fp16(h s + fp16(l s))
                  // is the reference's fp16(level * scale) up to rare near-ties
                  const uint32_t h = __byte_perm(lv_lo, lv_hi, sl);
                  const uint32_t l = __byte_perm(lw_lo, lw_hi, sl);
                  uint32_t ls;
                  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(ls) : "r"(l), "r"(sc));
                  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(fr[pr][d8]) : "r"(h), "r"(sc), "r"(ls));
                }
              }
              // a0 (dim g, slots 2t, 2t+1), a1 (dim g+8, same slots), a2 (dim
              // g, slots 2t+8, 2t+9), a3 (dim g+8, same slots)
              if constexpr (R == 8) mma_16816(acc[mt], fr[0][0], fr[0][1], fr[1][0], fr[1][1], cp0, cp1);
              mma_16816(acc[mt], fr[0][0], fr[0][1], fr[1][0], fr[1][1], bp0, bp1);
            }
          }
        }
      } else {
        const uint32_t vb = smem_u32(vdq_w) + kk_off * 128;
        for (int ks = 0; ks < SL / 16; ++ks) {
          // decode 16 tokens of the slice into this warp's fp16 staging tile
          if (compressed && vdec == 4) {
            // The 2-bit format with fp16 scales per 32 channels and no zeros
            // (the long TurboQuant-value workload): the same decoder with the
            // lane's word and scale offsets fixed for the launch and its two
            // scales in one 4-byte load.
            const int tk = lane >> 1, hw = lane & 1;
            const uint32_t sb = smem_u32(st);
            uint32_t w0, w1, w2, w3, s2;
            asm("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3) : "r"(sb + q4_word_off + ks * 512));
            asm("ld.shared.u32 %0, [%1];" : "=r"(s2) : "r"(sb + q4_scale_off + ks * 128));
            const uint32_t wrd[4] = {w0, w1, w2, w3};
            const float sca = __half2float(__ushort_as_half(static_cast<unsigned short>(s2 & 0xffffu)));
            const float scb = __half2float(__ushort_as_half(static_cast<unsigned short>(s2 >> 16)));
            const uint32_t lvb = smem_u32(&ms.lvpair[0]);
            uint64_t sa2, sb2;  // each scale twice, as a packed pair
            asm("mov.b64 %0, {%1, %1};" : "=l"(sa2) : "f"(sca));
            asm("mov.b64 %0, {%1, %1};" : "=l"(sb2) : "f"(scb));
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
              const int w = hw * 4 + wi;  // dims 16w .. 16w + 15
              const uint64_t s2 = wi < 2 ? sa2 : sb2;
              uint32_t h[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const uint32_t sh = j == 0 ? (wrd[wi] << 3) : (wrd[wi] >> (4 * j - 3));
                uint32_t a;
                asm("lop3.b32 %0, %1, 0x78, %2, 0xEA;" : "=r"(a) : "r"(sh), "r"(lvb));
                uint64_t x;
                asm("ld.shared.b64 %0, [%1];" : "=l"(x) : "r"(a));
                asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(x) : "l"(s2));
                float x0, x1;
                asm("mov.b64 {%0, %1}, %2;" : "=f"(x0), "=f"(x1) : "l"(x));
                h[j] = pack_h2(x0, x1);
              }
              *reinterpret_cast<uint4*>(vdq_w + vtile_addr(0, 16, tk, w * 16)) =
                  make_uint4(h[0], h[1], h[2], h[3]);
              *reinterpret_cast<uint4*>(vdq_w + vtile_addr(0, 16, tk, w * 16 + 8)) =
                  make_uint4(h[4], h[5], h[6], h[7]);
            }
          } else if (compressed && vdec == 1) {
            // 2-bit codes: lane = (token, half row); four 16-value words per
            // lane in one 16-byte load. Per nibble (two codes): one shift, one
            // three-input logic op forming the shared address of its level
            // pair (the 128-byte-aligned pair table), one 8-byte load, one
            // packed fp32 multiply (or multiply-add with the zero) and one
            // fp16 pack -- the reference's fp32 level * scale (+ zero),
            // rounded once to fp16.
            const uint8_t* sp = st + p.off_aux + TILE * p.v_words * 4;
            const float* zp = p.vz ? reinterpret_cast<const float*>(
                                         sp + TILE * p.v_groups * (p.vs_dt == SS_F32 ? 4 : 2))
                                   : nullptr;
            const int tk = lane >> 1, hw = lane & 1;
            const int tt = slice * SL + ks * 16 + tk;
            const uint4 wv = *reinterpret_cast<const uint4*>(st + p.off_aux + (tt * 8 + hw * 4) * 4);
            const uint32_t wrd[4] = {wv.x, wv.y, wv.z, wv.w};
            const uint32_t lvb = smem_u32(&ms.lvpair[0]);
            float sc[4], zr[4];
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
              const int gi = ((hw * 4 + wi) * 16) >> p.v_gshift;
              sc[wi] = p.vs_dt == SS_F32 ? reinterpret_cast<const float*>(sp)[tt * p.v_groups + gi]
                                         : h2f(reinterpret_cast<const uint16_t*>(sp)[tt * p.v_groups + gi]);
              zr[wi] = zp ? zp[tt * p.v_groups + gi] : 0.f;
            }
            auto decode = [&](auto with_zero) {
#pragma unroll
              for (int wi = 0; wi < 4; ++wi) {
                const int w = hw * 4 + wi;  // dims 16w .. 16w + 15
                uint32_t h[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const uint32_t sh = j == 0 ? (wrd[wi] << 3) : (wrd[wi] >> (4 * j - 3));
                  uint32_t a;
                  asm("lop3.b32 %0, %1, 0x78, %2, 0xEA;" : "=r"(a) : "r"(sh), "r"(lvb));  // (sh & 0x78) | lvb
                  float x0, x1;
                  asm("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(x0), "=f"(x1) : "r"(a));
                  if constexpr (decltype(with_zero)::value) mul_add_f32x2(x0, x1, sc[wi], zr[wi]);
                  else mul_f32x2(x0, x1, sc[wi]);
                  h[j] = pack_h2(x0, x1);
                }
                *reinterpret_cast<uint4*>(vdq_w + vtile_addr(0, 16, tk, w * 16)) =
                    make_uint4(h[0], h[1], h[2], h[3]);
                *reinterpret_cast<uint4*>(vdq_w + vtile_addr(0, 16, tk, w * 16 + 8)) =
                    make_uint4(h[4], h[5], h[6], h[7]);
              }
            };
            if (zp) decode(std::true_type{});
            else decode(std::false_type{});
          } else if (compressed && vdec == 2) {
            // block-VQ values: lane = (token, half row); one index byte per
            // block, one table row of v_bd fp16 per block
            const int tk = lane >> 1, hw = lane & 1;
            const int tt = slice * SL + ks * 16 + tk;
            const uint8_t* ir = st + p.off_aux + tt * p.v_nb;
            const uint16_t* vt = reinterpret_cast<const uint16_t*>(smem + p.off_vtab);
            if (p.v_bd == 4) {
              const uint4 c4 = *reinterpret_cast<const uint4*>(ir + hw * 16);
              const uint32_t cw4[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
              for (int w = 0; w < 4; ++w) {
#pragma unroll
                for (int j = 0; j < 4; j += 2) {
                  const int b = hw * 16 + w * 4 + j;
                  const uint32_t c0 = (cw4[w] >> (8 * j)) & 255u, c1 = (cw4[w] >> (8 * j + 8)) & 255u;
                  const uint2 e0 = *reinterpret_cast<const uint2*>(vt + ((b << 8) + c0) * 4);
                  const uint2 e1 = *reinterpret_cast<const uint2*>(vt + (((b + 1) << 8) + c1) * 4);
                  *reinterpret_cast<uint4*>(vdq_w + vtile_addr(0, 16, tk, b * 4)) =
                      make_uint4(e0.x, e0.y, e1.x, e1.y);
                }
              }
            } else if (p.v_bd == 8) {
              const uint2 c2 = *reinterpret_cast<const uint2*>(ir + hw * 8);
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int b = hw * 8 + j;
                const uint32_t c = ((j < 4 ? c2.x : c2.y) >> (8 * (j & 3))) & 255u;
                *reinterpret_cast<uint4*>(vdq_w + vtile_addr(0, 16, tk, b * 8)) =
                    *reinterpret_cast<const uint4*>(vt + ((b << 8) + c) * 8);
              }
            } else {
              const uint32_t c1 = *reinterpret_cast<const uint32_t*>(ir + hw * 4);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int b = hw * 4 + j;
                const uint32_t c = (c1 >> (8 * j)) & 255u;
                const uint16_t* e = vt + ((b << 8) + c) * 16;
                *reinterpret_cast<uint4*>(vdq_w + vtile_addr(0, 16, tk, b * 16)) =
                    *reinterpret_cast<const uint4*>(e);
                *reinterpret_cast<uint4*>(vdq_w + vtile_addr(0, 16, tk, b * 16 + 8)) =
                    *reinterpret_cast<const uint4*>(e + 8);
              }
            }
          } else if (compressed) {
            const uint32_t* words = reinterpret_cast<const uint32_t*>(st + p.off_aux);
            const uint8_t* sp = st + p.off_aux + TILE * p.v_words * 4;
            const float* zp = p.vz ? reinterpret_cast<const float*>(
                                         sp + TILE * p.v_groups * (p.vs_dt == SS_F32 ? 4 : 2))
                                   : nullptr;
            const int vpw = p.v_bits == 3 ? 10 : 32 / p.v_bits;
            const uint32_t msk = (1u << p.v_bits) - 1u;
            for (int e = lane; e < 16 * (D / 8); e += 32) {
              const int tk = e / (D / 8), ch = e - tk * (D / 8);
              const int tt = slice * SL + ks * 16 + tk;
              const int gi = (ch * 8) / p.v_group;
              const float s_ = p.vs_dt == SS_F32
                                   ? reinterpret_cast<const float*>(sp)[tt * p.v_groups + gi]
                                   : h2f(reinterpret_cast<const uint16_t*>(sp)[tt * p.v_groups + gi]);
              const float z_ = zp ? zp[tt * p.v_groups + gi] : 0.f;
              float vals[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int c = ch * 8 + j;
                const uint32_t code = (words[tt * p.v_words + c / vpw] >> ((c % vpw) * p.v_bits)) & msk;
                float x = __fmul_rn(ms.levels[code], s_);
                if (zp) x = __fadd_rn(x, z_);
                vals[j] = x;
              }
              uint4 pk;
              pk.x = pack_h2(vals[0], vals[1]);
              pk.y = pack_h2(vals[2], vals[3]);
              pk.z = pack_h2(vals[4], vals[5]);
              pk.w = pack_h2(vals[6], vals[7]);
              *reinterpret_cast<uint4*>(vdq_w + vtile_addr(0, 16, tk, ch * 8)) = pk;
            }
          } else {
            for (int e = lane; e < 16 * (D / 8); e += 32) {
              const int tk = e / (D / 8), ch = e - tk * (D / 8);
              const int tt = slice * SL + ks * 16 + tk;
              uint4 pk = make_uint4(0, 0, 0, 0);
              if (tt < len)
                pk = *reinterpret_cast<const uint4*>(p.v_tail + pair * p.tail_ps + (t0 + tt) * D + ch * 8);
              *reinterpret_cast<uint4*>(vdq_w + vtile_addr(0, 16, tk, ch * 8)) = pk;
            }
          }
          __syncwarp();
          uint32_t b0, b1, c0 = 0, c1 = 0;
          ldsm_x2_trans(pw_addr + ks * 256, b0, b1);
          if constexpr (R == 8) ldsm_x2_trans(pwl_addr + ks * 256, c0, c1);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const uint32_t col = (mt >> 2) * (16 * 128) + ((((2 * mt + dsel) & 7) ^ mj) << 4);
            uint32_t x0, x1, x2, x3;
            ldsm_x4_trans(vb + col, x0, x1, x2, x3);
            if constexpr (R == 8) mma_16816(acc[mt], x0, x1, x2, x3, c0, c1);
            mma_16816(acc[mt], x0, x1, x2, x3, b0, b1);
          }
          __syncwarp();
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[s]);
    }

    // ---------------------------------------------- merge the warps of this CTA
    float l_w[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float v = l_l[r];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      l_w[r] = v;
    }
    named_bar_sync(1, (CW * 32));  // every warp is done with the LUT: reuse it as scratch
    float* wo = lut;                                  // [8][R][D]
    float* wm = lut + CW * R * D;         // [8][R]
    float* wl = wm + CW * R;              // [8][R]
    // merged unit rows for finalisation, after the per-warp scratch, then the
    // merge weights (per warp, or per cross-CTA partial, and row)
    float (*mo)[D] = reinterpret_cast<float (*)[D]>(lut + CW * R * (D + 2));
    float* wt = lut + CW * R * (D + 2) + R * D;
    if constexpr (R <= 4) {
      // add the lo-half columns 4..7 (lanes t + 2) to their rows' columns
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[mt][i] += __shfl_xor_sync(0xffffffffu, acc[mt][i], 2);
    }
    {
      const int n0 = 2 * (lane & 3);
      const int m0 = lane >> 2;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        if (n0 < R) {
          wo[(warp * R + n0) * D + mt * 16 + m0] = acc[mt][0];
          wo[(warp * R + n0) * D + mt * 16 + m0 + 8] = acc[mt][2];
        }
        if (n0 + 1 < R) {
          wo[(warp * R + n0 + 1) * D + mt * 16 + m0] = acc[mt][1];
          wo[(warp * R + n0 + 1) * D + mt * 16 + m0 + 8] = acc[mt][3];
        }
      }
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < R; ++r) { wm[warp * R + r] = m_w[r]; wl[warp * R + r] = l_w[r]; }
      }
    }
    if (ctid == 0) ms.is_last = 0;
    named_bar_sync(1, (CW * 32));
    // one weight per (warp, row): e^(m_w - m*)
    if (ctid < CW * R) {
      const int w = ctid / R, r = ctid - w * R;
      float mstar = -INFINITY;
#pragma unroll
      for (int x = 0; x < CW; ++x) mstar = fmaxf(mstar, wm[x * R + r]);
      const float mg = wm[w * R + r];
      wt[w * R + r] = (mg == -INFINITY) ? 0.f : fast_exp2((mg - mstar) * kLog2e);
      if (w == 0) ms.mrow[r] = mstar;
    }
    named_bar_sync(1, (CW * 32));
    for (int e = ctid; e < R * D; e += (CW * 32)) {
      const int r = e / D, j = e - r * D;
      float O = 0.f;
#pragma unroll
      for (int w = 0; w < CW; ++w) O = fmaf(wo[(w * R + r) * D + j], wt[w * R + r], O);
      mo[r][j] = O;
    }
    if (ctid < R) {
      float L = 0.f;
#pragma unroll
      for (int w = 0; w < CW; ++w) L = fmaf(wl[w * R + ctid], wt[w * R + ctid], L);
      ms.lrow[ctid] = L;
    }
    named_bar_sync(1, (CW * 32));

    // ---------------------------------------------- unit finalisation
    const int64_t first = cta_of(sched, u * p.tpu);
    const int64_t last = cta_of(sched, (u + 1) * p.tpu - 1);
    const int ncov = static_cast<int>(last - first + 1);
    const int row_floats = D + 2;
    bool do_final = true;
    if (ncov > 1) {
      float* slot = p.slots + ((size_t)u * p.max_cov + (cta - first)) * R * row_floats;
      for (int e = ctid; e < R * row_floats; e += (CW * 32)) {
        const int r = e / row_floats, j = e - r * row_floats;
        slot[e] = j < D ? mo[r][j] : (j == D ? ms.mrow[r] : ms.lrow[r]);
      }
      named_bar_sync(1, (CW * 32));
      if (ctid == 0) {
        // the barrier orders every thread's slot writes before this
        // release; its acquire half makes the other partials visible to the
        // CTA that arrives last
        int prev;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                     : "=r"(prev) : "l"(p.counters + u) : "memory");
        if (prev == ncov - 1) {
          ms.is_last = 1;
          p.counters[u] = 0;  // leave the counter ready for the next launch
        }
      }
      named_bar_sync(1, (CW * 32));
      do_final = ms.is_last != 0;
      if (do_final) {
        __threadfence();
        const float* base = p.slots + (size_t)u * p.max_cov * R * row_floats;
        // row maxima over the partials, then one weight per (partial, row)
        if (ctid < R) {
          float mstar = -INFINITY;
#pragma unroll 4
          for (int g = 0; g < ncov; ++g)
            mstar = fmaxf(mstar, __ldcg(base + ((size_t)g * R + ctid) * row_floats + D));
          ms.mrow[ctid] = mstar;
        }
        named_bar_sync(1, (CW * 32));
        for (int e = ctid; e < ncov * R; e += (CW * 32)) {
          const int r = e % R;
          const float mg = __ldcg(base + (size_t)e * row_floats + D);
          wt[e] = (mg == -INFINITY) ? 0.f : fast_exp2((mg - ms.mrow[r]) * kLog2e);
        }
        named_bar_sync(1, (CW * 32));
        for (int e = ctid; e < R * D; e += (CW * 32)) {
          const int r = e / D, j = e - r * D;
          float O = 0.f;
#pragma unroll 4
          for (int g = 0; g < ncov; ++g)
            O = fmaf(__ldcg(base + ((size_t)g * R + r) * row_floats + j), wt[g * R + r], O);
          mo[r][j] = O;
        }
        if (ctid < R) {
          float L = 0.f;
          for (int g = 0; g < ncov; ++g)
            L = fmaf(__ldcg(base + ((size_t)g * R + ctid) * row_floats + D + 1), wt[g * R + ctid], L);
          ms.lrow[ctid] = L;
        }
        named_bar_sync(1, (CW * 32));
      }
    }
    // fp16 output rows without a value rotation, 16-byte aligned: 8 elements
    // per thread in one 16-byte store (fewer, larger writes, which matters
    // when the output lives in page-locked host memory)
    const bool vec_out = do_final && !p.part_out && !p.v_rot && p.odt == SS_F16 &&
                         (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 &&
                         ((p.o_sb | p.o_sh | p.o_st) & 7) == 0;
    if (vec_out) {
      for (int e8 = ctid; e8 < R * D / 8; e8 += (CW * 32)) {
        const int r = e8 / (D / 8), j0 = (e8 - r * (D / 8)) * 8;
        const int rr = rg * R + r;
        if (rr >= rows_valid) continue;
        const int rep = rr / p.tq, tqi = rr - rep * p.tq;
        const int qh = hh * p.nrep + rep;
        const float inv = ms.lrow[r] > 0.f ? 1.f / ms.lrow[r] : 0.f;
        uint4 h;
        h.x = pack_h2(mo[r][j0] * inv, mo[r][j0 + 1] * inv);
        h.y = pack_h2(mo[r][j0 + 2] * inv, mo[r][j0 + 3] * inv);
        h.z = pack_h2(mo[r][j0 + 4] * inv, mo[r][j0 + 5] * inv);
        h.w = pack_h2(mo[r][j0 + 6] * inv, mo[r][j0 + 7] * inv);
        *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(p.out) + bb * p.o_sb + qh * p.o_sh +
                                  tqi * p.o_st + j0) = h;
      }
    } else if (do_final) {
      for (int e = ctid; e < R * D; e += (CW * 32)) {
        const int r = e / D, j = e - r * D;
        const int rr = rg * R + r;
        if (rr >= rows_valid) continue;
        const int rep = rr / p.tq, tqi = rr - rep * p.tq;
        const int qh = hh * p.nrep + rep;
        if (p.part_out) {
          float* row = p.part_out + (((int64_t)bb * p.hq + qh) * p.tq + tqi) * (D + 2);
          row[j] = mo[r][j];
          if (j == 0) { row[D] = ms.mrow[r]; row[D + 1] = ms.lrow[r]; }
        } else {
          const float inv = ms.lrow[r] > 0.f ? 1.f / ms.lrow[r] : 0.f;
          float v;
          if (p.v_rot) {
            float a = 0.f;
            for (int i = 0; i < D; ++i) a = fmaf(mo[r][i], __ldg(p.v_rot + i * D + j), a);
            v = a * inv;
          } else {
            v = mo[r][j] * inv;
          }
          store_from_f32(p.out, p.odt, bb * p.o_sb + qh * p.o_sh + tqi * p.o_st + j, v);
        }
      }
    }
    tau = u_end;
  }
  // a table copy still in flight after a give-up must land before the CTA
  // exits (its shared memory is then handed to other CTAs)
  if (ctid == 0 && lut_out && !mbar_wait_bounded(&lut_bar, lut_phase, p.wait_ns))
    report_wait_failure(p.err, p.sink, 8);
}

// ------------------------------------------------------------------ merge
// Split-KV merge of per-shard (o, m, l) rows (one CTA per row).
__global__ void lse_merge_kernel(const float* parts, int n_parts, int64_t rows, int d,
                                 const float* v_rot, void* out, int odt, int64_t out_stride) {
  __shared__ float s_o[512];
  __shared__ float s_w[64];
  const int64_t row = blockIdx.x;
  const int rf = d + 2;
  float mstar = -INFINITY;
  for (int g = 0; g < n_parts; ++g) mstar = fmaxf(mstar, parts[((int64_t)g * rows + row) * rf + d]);
  if (threadIdx.x < n_parts) {
    const float mg = parts[((int64_t)threadIdx.x * rows + row) * rf + d];
    s_w[threadIdx.x] = (mg == -INFINITY) ? 0.f : exp2f((mg - mstar) * kLog2e);
  }
  __syncthreads();
  float L = 0.f;
  for (int g = 0; g < n_parts; ++g) L += parts[((int64_t)g * rows + row) * rf + d + 1] * s_w[g];
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    float o = 0.f;
    for (int g = 0; g < n_parts; ++g) o = fmaf(parts[((int64_t)g * rows + row) * rf + j], s_w[g], o);
    s_o[j] = o * inv;
  }
  __syncthreads();
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    float v = s_o[j];
    if (v_rot) {
      float a = 0.f;
      for (int i = 0; i < d; ++i) a = fmaf(s_o[i], v_rot[i * d + j], a);
      v = a;
    }
    store_from_f32(out, odt, row * out_stride + j, v);
  }
}

// ------------------------------------------------------------------ host plan
struct Plan {
  int R, cw, tile, n_rg, n_ct, n_tt, tpu, grid, stages, max_cov, v_words, v_groups, w_unit;
  int64_t total_tiles, n_units;
  uint32_t stage_bytes, off_idx, off_aux, off_vdq, off_lut, off_p, off_misc, off_vtab, v_tile_bytes;
  uint32_t off_plo;
  size_t smem;
  size_t ws_bytes, off_counters, off_slots, off_lut_g, lut_unit_bytes;
};

constexpr size_t kSmemBudget = 226 * 1024;  // leaves room for static barriers

int make_plan_r(const ss_decode_args* a, Plan& pl, int r_cap, int cw) {
  SS_REQUIRE(a, "ss_decode_attn: null args");
  SS_REQUIRE(a->d == 64 || a->d == 128, "ss_decode_attn: head_dim must be 64 or 128");
  SS_REQUIRE(a->bd > 0 && a->bd <= 16 && a->d % a->bd == 0, "ss_decode_attn: bad block_dim");
  SS_REQUIRE(a->k >= 1 && a->k <= 256, "ss_decode_attn: k must be in [1, 256]");
  SS_REQUIRE(a->hkv > 0 && a->hq % a->hkv == 0, "ss_decode_attn: hq must be a multiple of hkv");
  SS_REQUIRE(a->b >= 0 && a->tq >= 1 && a->tc >= 0 && a->ttail >= 0,
             "ss_decode_attn: bad batch / lengths");
  SS_REQUIRE(a->vfmt == SS_V_F16 || a->vfmt == SS_V_QUANT || a->vfmt == SS_V_VQ,
             "ss_decode_attn: bad vfmt");
  if (a->vfmt == SS_V_VQ)
    SS_REQUIRE(a->d == 128 && (a->v_bd == 4 || a->v_bd == 8 || a->v_bd == 16) && a->v_k >= 1 &&
                   a->v_k <= 256,
               "ss_decode_attn: VQ values need head_dim 128, v_bd in {4, 8, 16}, v_k <= 256");
  SS_REQUIRE(a->n_heavy >= 0 && a->n_heavy <= 32, "ss_decode_attn: n_heavy must be <= 32");
  const int nb = a->d / a->bd;
  const int nrep = a->hq / a->hkv;
  const int rows = nrep * a->tq;
  int R = rows >= 5 ? 8 : (rows >= 3 ? 4 : (rows == 2 ? 2 : 1));
  while (R > r_cap || (R > 1 && (size_t)nb * a->k * R * 4 > 128 * 1024)) R >>= 1;
  pl.R = R;
  pl.tile = 128;
  SS_REQUIRE(nb % 2 == 0 && nb <= 128, "ss_decode_attn: n_blocks must be even and <= 128");
  pl.n_rg = (rows + R - 1) / R;
  pl.n_ct = static_cast<int>((a->tc + pl.tile - 1) / pl.tile);
  pl.n_tt = static_cast<int>((a->ttail + pl.tile - 1) / pl.tile);
  pl.tpu = pl.n_ct + pl.n_tt;
  pl.n_units = (int64_t)a->b * a->hkv * pl.n_rg;
  pl.total_tiles = pl.n_units * pl.tpu;
  const int sms = sm_count();
  int64_t g = pl.total_tiles < sms ? pl.total_tiles : sms;
  if (a->max_ctas > 0 && g > a->max_ctas) g = a->max_ctas;
  pl.grid = static_cast<int>(g < 1 ? 1 : g);
  // a unit boundary inside a CTA's range (merge, cross-CTA publish, table
  // reload) costs about as much as 14 tiles of streaming (measured on the 16 x 8192-token batched decode)
  pl.w_unit = pl.n_units > 1 ? 14 : 0;
  {
    // CTAs covering one unit: bounded by the shortest non-empty range (an
    // empty range is a cost share inside a boundary's gap and covers no unit)
    const Sched sc = make_sched(pl.total_tiles, pl.tpu, pl.w_unit, pl.grid);
    int64_t shortest = pl.total_tiles;
    for (int k = 0; k < pl.grid; ++k) {
      const int64_t len = range_start(sc, k + 1) - range_start(sc, k);
      if (len > 0 && len < shortest) shortest = len;
    }
    pl.max_cov = static_cast<int>(pl.tpu / (shortest > 0 ? shortest : 1)) + 2;
    if (pl.max_cov > pl.grid) pl.max_cov = pl.grid;
  }
  pl.v_words = 0;
  pl.v_groups = 0;
  int sbytes = 0;
  if (a->vfmt == SS_V_QUANT) {
    SS_REQUIRE(a->v_bits >= 2 && a->v_bits <= 4, "ss_decode_attn: v_bits must be 2..4");
    SS_REQUIRE(a->v_group >= 8 && a->v_group % 8 == 0 && a->d % a->v_group == 0,
               "ss_decode_attn: v_group must be a multiple of 8 dividing head_dim");
    SS_REQUIRE(a->v_scale_dtype == SS_F32 || a->v_scale_dtype == SS_F16,
               "ss_decode_attn: bad scale dtype");
    pl.v_words = a->v_bits == 3 ? (a->d + 9) / 10 : a->d / (32 / a->v_bits);
    pl.v_groups = a->d / a->v_group;
    sbytes = a->v_scale_dtype == SS_F32 ? 4 : 2;
  }
  const uint32_t T = pl.tile;
  const uint32_t vbytes = a->vfmt == SS_V_F16 ? T * a->d * 2 : 0;
  pl.off_idx = vbytes;
  pl.off_aux = (vbytes + T * nb + 127) & ~127u;
  uint32_t aux = 0;
  if (a->vfmt == SS_V_QUANT) {
    aux += T * pl.v_words * 4 + T * pl.v_groups * sbytes;
    if (a->v_zeros) aux += T * pl.v_groups * 4;
  } else if (a->vfmt == SS_V_VQ) {
    aux += T * (a->d / a->v_bd);
  }
  pl.v_tile_bytes = aux;
  aux += T * a->n_heavy * a->bd * 2;
  pl.stage_bytes = (pl.off_aux + aux + 1023) & ~1023u;
  size_t fixed = 0;
  // per-warp fp16 value slices (16 tokens) for the quantized path
  const size_t vdq = (a->vfmt != SS_V_F16) ? (size_t)cw * 16 * a->d * 2 : 0;
  // VQ value centroids [nb_v][256][bd_v] fp16, resident for the whole launch
  const size_t vtab = (a->vfmt == SS_V_VQ) ? (size_t)a->d * 256 * 2 : 0;
  // the LUT region doubles as the per-warp merge scratch at unit ends
  size_t lut = (size_t)nb * a->k * R * 4;
  // per-warp merge scratch + the merged rows of the unit + merge weights
  // (per warp or per cross-CTA partial, and row)
  const size_t n_wt = std::max<size_t>((size_t)cw, (size_t)pl.max_cov);
  const size_t scratch = (size_t)cw * R * (a->d + 2) * 4 + (size_t)R * a->d * 4 + n_wt * R * 4;
  if (lut < scratch) lut = scratch;
  size_t pbytes = (size_t)cw * slice_tokens(R) * 16;  // per-warp P slice [tokens][8] fp16
  // 8-row units keep the lo halves of P in a second slice per warp: in the
  // unit's query rows of Misc (4 KB, free during the tile loop when there is
  // no fp16 tail to score), else in a region of their own
  const bool plo_own = R == 8 && (a->ttail > 0 || (size_t)cw * slice_tokens(R) * 16 > sizeof(float) * 8 * 128);
  const size_t plo = plo_own ? pbytes : 0;
  pbytes += plo;
  fixed = vdq + vtab + ((lut + 127) & ~size_t(127)) + pbytes + ((sizeof(Misc) + 127) & ~size_t(127)) + 1024;
  if (fixed + 2 * (size_t)pl.stage_bytes > kSmemBudget)
    return fail(SS_ERR_UNSUPPORTED, "ss_decode_attn: configuration exceeds shared memory");
  int stages = static_cast<int>((kSmemBudget - fixed) / pl.stage_bytes);
  if (stages > (cw == 16 ? 8 : 6)) stages = cw == 16 ? 8 : 6;
  // The consumer warps form tile groups that take tiles round robin; a warp may
  // only wait for the barrier phase right after the one it consumed last,
  // which holds when the stage count is a multiple of the number of groups.
  const int tgroups = cw * slice_tokens(R) / static_cast<int>(T);  // warps / warps per tile
  stages -= stages % tgroups;
  // 12 consumer warps only pay off with two free stages beyond the three in use
  if (stages < tgroups || (cw > 8 && stages < tgroups + 2))
    return fail(SS_ERR_UNSUPPORTED, "ss_decode_attn: configuration exceeds shared memory");
  pl.cw = cw;
  pl.stages = stages;
  size_t off = (size_t)stages * pl.stage_bytes;
  pl.off_vdq = static_cast<uint32_t>(off);
  off += vdq;
  pl.off_vtab = static_cast<uint32_t>(off);
  off += vtab;
  pl.off_lut = static_cast<uint32_t>(off);
  off += (lut + 127) & ~size_t(127);
  pl.off_p = static_cast<uint32_t>(off);
  pl.off_plo = plo_own ? static_cast<uint32_t>(off + (pbytes - plo)) : 0u;
  off += pbytes;
  pl.off_misc = static_cast<uint32_t>(off);
  off += (sizeof(Misc) + 127) & ~size_t(127);
  pl.smem = off + 1024;
  // workspace: [error word | counters | partial slots]
  pl.off_counters = 256;
  pl.off_slots = (pl.off_counters + (size_t)pl.n_units * 4 + 255) & ~size_t(255);
  pl.lut_unit_bytes = (size_t)nb * a->k * R * 4;
  pl.off_lut_g = (pl.off_slots + (size_t)pl.n_units * pl.max_cov * R * (a->d + 2) * 4 + 255) &
                 ~size_t(255);
  pl.ws_bytes = pl.off_lut_g + (size_t)pl.n_units * pl.lut_unit_bytes;
  return SS_OK;
}

// Largest row group that fits: 8 query rows per unit need a 128 KB table next
// to the stage ring; when that does not fit (wide stages, or the value
// centroid table of VQ values) the rows are split into smaller groups, each of
// which streams the unit once.
// 12 consumer warps (more latency hiding for the table gather) when six
// stages fit, i.e. for compact value formats; 8 warps with 4 stages otherwise.
int make_plan(const ss_decode_args* a, Plan& pl) {
  int rc = SS_ERR_UNSUPPORTED;
  for (int r_cap = 8;;) {
    // 16 consumer warps only for the lean 2-bit-value kernel (4 rows, 16
    // key blocks, compressed tokens only): its per-token work is latency
    // bound and the small stages leave room for a fourth tile group
    const bool q16 = a->vfmt == SS_V_QUANT && a->d == 128 && a->v_bits == 2 &&
                     a->v_group == 32 && a->v_scale_dtype == SS_F16 && !a->v_zeros &&
                     a->d / a->bd == 16 && a->k == 256 && a->n_heavy == 0 && a->ttail == 0 &&
                     !a->causal && a->mask == nullptr && a->hq / a->hkv * a->tq == 4;
    for (int cw : {16, 12, 8}) {
      if (cw == 16 && !q16) continue;
      rc = make_plan_r(a, pl, r_cap, cw);
      if (rc != SS_ERR_UNSUPPORTED) return rc;
    }
    if (pl.R <= 1) break;
    r_cap = pl.R / 2;  // halve the row group (the stream is read once per group)
  }
  return rc;
}

template <int R, int D>
int launch_decode(const DecodeParams& p, const CUtensorMap& mv, const CUtensorMap& mvt,
                  size_t smem, int cw, cudaStream_t st) {
  const dim3 lgrid(static_cast<unsigned>(p.n_units), (p.nb + kLutBlocks - 1) / kLutBlocks);
  // Same shared-memory carveout as the decode kernel: no reconfiguration
  // between the two launches of every step.
  static bool carveout_set = false;
  if (!carveout_set) {
    cudaFuncSetAttribute(lut_kernel<R, 8>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(lut_kernel<R, 4>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(lut_kernel<R, 0>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    carveout_set = true;
  }
  if (p.rot_k == nullptr && (p.bd == 8 || p.bd == 4) && p.k <= 256) {
    const dim3 bgrid(static_cast<unsigned>(p.nb), static_cast<unsigned>(p.lut_groups + p.app_groups));
    // programmatic dependent of the previous kernel in the stream (the
    // kernel waits for it before touching anything but codec state)
    cudaLaunchConfig_t lc = {};
    lc.gridDim = bgrid;
    lc.blockDim = dim3(256);
    lc.stream = st;
    cudaLaunchAttribute la[1];
    la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    la[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = la;
    lc.numAttrs = 1;
    const cudaError_t le = p.bd == 8 ? cudaLaunchKernelEx(&lc, lut_block_kernel<R, 8>, p)
                                     : cudaLaunchKernelEx(&lc, lut_block_kernel<R, 4>, p);
    if (le != cudaSuccess)
      return fail(SS_ERR_CUDA, std::string("ss_decode_attn: table launch: ") + cudaGetErrorString(le));
  } else if (p.bd == 8) {
    lut_kernel<R, 8><<<lgrid, kLutThreads, 0, st>>>(p);
  } else if (p.bd == 4) {
    lut_kernel<R, 4><<<lgrid, kLutThreads, 0, st>>>(p);
  } else {
    lut_kernel<R, 0><<<lgrid, kLutThreads, 0, st>>>(p);
  }
  int rc = check_launch("ss_decode_attn (tables)");
  if (rc != SS_OK) return rc;
  const bool nb16 = p.nb == 16 && p.k == 256;
  // the warp-MMA heavy-block variant only where it can apply (it holds the
  // query fragments in registers for the whole unit)
  const int hd = p.n_heavy * p.bd;
  const bool hv = (R == 4 || R == 8) && D == 128 && p.n_heavy > 0 && hd % 16 == 0 && hd <= 64;
  constexpr bool kHv = (R == 4 || R == 8) && D == 128;
  auto kern = cw == 12 ? (nb16 ? decode_attn_kernel<R, D, 16, 12, false> : decode_attn_kernel<R, D, 0, 12, false>)
                       : (nb16 ? decode_attn_kernel<R, D, 16, 8, false> : decode_attn_kernel<R, D, 0, 8, false>);
  if (kHv && hv)
    kern = cw == 12 ? (nb16 ? decode_attn_kernel<R, D, 16, 12, kHv> : decode_attn_kernel<R, D, 0, 12, kHv>)
                    : (nb16 ? decode_attn_kernel<R, D, 16, 8, kHv> : decode_attn_kernel<R, D, 0, 8, kHv>);
  // Lean variants for the two streaming formats of the batched workloads
  // (compressed tokens only, no heavy blocks, no masks): every other branch
  // is compiled out, which frees registers and issue slots per tile.
  bool lean16 = false;
  if constexpr ((R == 4 || R == 8) && D == 128) {
    const bool plain = nb16 && !hv && p.n_heavy == 0 && p.n_tt == 0 && !p.causal && p.mask == nullptr;
    if constexpr (R == 4) {
      if (plain && p.vdec == 0 && cw == 8) kern = decode_attn_kernel<R, D, 16, 8, false, 1>;
      if (plain && p.vdec == 4 && cw == 12) kern = decode_attn_kernel<R, D, 16, 12, false, 2>;
      if (plain && p.vdec == 4 && cw == 16) {
        kern = decode_attn_kernel<R, D, 16, 16, false, 2>;
        lean16 = true;
      }
    } else {
      // fp16 values with heavy (fp16 pass-through) key blocks on warp MMAs, 8
      // rows (the long mixed-precision sequence), compressed tokens only, no masks
      if (nb16 && hv && p.vdec == 0 && p.n_tt == 0 && !p.causal && p.mask == nullptr && cw == 8)
        kern = decode_attn_kernel<R, D, 16, 8, kHv, 3>;
    }
  }
  // block-VQ values (both K and V as block VQ, the model harness's cache),
  // compressed tokens only, no heavy blocks, no masks
  if constexpr ((R == 2 || R == 4) && D == 128) {
    if (!nb16 && p.vdec == 2 && p.n_heavy == 0 && p.n_tt == 0 && !p.causal && p.mask == nullptr &&
        cw == 8)
      kern = decode_attn_kernel<R, D, 0, 8, false, 4>;
  }
  if (cw == 16 && !lean16)
    return fail(SS_ERR_UNSUPPORTED, "ss_decode_attn: 16 consumer warps need the lean 2-bit kernel");
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess)
    return fail(SS_ERR_CUDA, std::string("ss_decode_attn: smem attribute: ") + cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(cw * 32 + 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, p, mv, mvt);
  if (e != cudaSuccess)
    return fail(SS_ERR_CUDA, std::string("ss_decode_attn: launch: ") + cudaGetErrorString(e));
  return check_launch("ss_decode_attn");
}

int run_decode(const ss_decode_args* a, float* part_out, void* stream,
               const char* name = nullptr) {
  Plan pl;
  int rc = make_plan(a, pl);
  if (rc != SS_OK) return rc;
  SS_REQUIRE(a->q && a->centroids && a->out || part_out, "ss_decode_attn: null pointer");
  SS_REQUIRE(a->tc == 0 || a->idx, "ss_decode_attn: idx is null");
  SS_REQUIRE(a->ttail == 0 || (a->k_tail && a->v_tail), "ss_decode_attn: tail is null");
  SS_REQUIRE(a->n_heavy == 0 || (a->heavy && a->kheavy), "ss_decode_attn: heavy data is null");
  SS_REQUIRE(a->tc == 0 || a->vfmt != SS_V_F16 || a->v, "ss_decode_attn: v is null");
  SS_REQUIRE(a->tc == 0 || a->vfmt != SS_V_QUANT || (a->vq && a->v_scales),
             "ss_decode_attn: quantized values are null");
  SS_REQUIRE(a->tc == 0 || a->vfmt != SS_V_VQ || (a->v_idx && a->v_cents),
             "ss_decode_attn: VQ value indices / centroids are null");
  cudaStream_t st = as_stream(stream);
  const int64_t n_pairs = (int64_t)a->b * a->hkv;
  if (pl.total_tiles == 0 || n_pairs == 0) return SS_OK;  // caller zero-fills empty caches
  if (!a->workspace || a->workspace_bytes < pl.ws_bytes)
    return fail(SS_ERR_WORKSPACE, "ss_decode_attn: workspace missing or too small");
  const int nb = a->d / a->bd;
  const int64_t rows_cap = a->v_pair_stride / a->d;
  // 16-byte alignment of every bulk-copied row block
  auto aligned = [](const void* ptr, int64_t pair_stride_bytes) {
    return reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && pair_stride_bytes % 16 == 0;
  };
  if (a->tc > 0) {
    SS_REQUIRE(aligned(a->idx, a->idx_pair_stride),
               "ss_decode_attn: idx base / pair stride must be 16-byte aligned");
    if (a->vfmt == SS_V_QUANT) {
      const int sb = a->v_scale_dtype == SS_F32 ? 4 : 2;
      SS_REQUIRE(aligned(a->vq, a->vq_pair_stride * 4) &&
                     aligned(a->v_scales, a->vs_pair_stride * sb) &&
                     (!a->v_zeros || aligned(a->v_zeros, a->vz_pair_stride * 4)),
                 "ss_decode_attn: quantized value streams must be 16-byte aligned");
    }
    if (a->vfmt == SS_V_VQ) {
      SS_REQUIRE(aligned(a->v_idx, a->vi_pair_stride) && aligned(a->v_cents, 0),
                 "ss_decode_attn: VQ value indices / centroids must be 16-byte aligned");
      SS_REQUIRE(a->vi_pair_stride / (a->d / a->v_bd) >= (int64_t)pl.n_ct * pl.tile,
                 "ss_decode_attn: VQ value rows per pair must cover whole 128-token tiles");
    }
    if (a->n_heavy)
      SS_REQUIRE(aligned(a->kheavy, a->kheavy_pair_stride * 2),
                 "ss_decode_attn: heavy key stream must be 16-byte aligned");
  }
  if (a->ttail > 0)
    SS_REQUIRE(aligned(a->k_tail, a->tail_pair_stride * 2) &&
                   aligned(a->v_tail, a->tail_pair_stride * 2),
               "ss_decode_attn: tail streams must be 16-byte aligned");
  CUtensorMap mv{}, mvt{};
  if (a->vfmt == SS_V_F16 && a->tc > 0) {
    SS_REQUIRE(a->v_pair_stride % a->d == 0 && rows_cap >= a->tc, "ss_decode_attn: bad v stride");
    const CUtensorMap* m = tmap_3d_f16_sw128(a->v, a->d, rows_cap, n_pairs,
                                             a->v_pair_stride * 2, 64, pl.tile);
    if (!m) return SS_ERR_CUDA;
    mv = *m;
  }
  if (a->ttail > 0) {
    SS_REQUIRE(a->tail_pair_stride % a->d == 0 && a->tail_pair_stride / a->d >= a->ttail,
               "ss_decode_attn: bad tail stride");
    if (a->vfmt == SS_V_F16) {
      const CUtensorMap* m = tmap_3d_f16_sw128(a->v_tail, a->d, a->tail_pair_stride / a->d,
                                               n_pairs, a->tail_pair_stride * 2, 64, pl.tile);
      if (!m) return SS_ERR_CUDA;
      mvt = *m;
    }
  }
  DecodeParams p{};
  p.b = a->b; p.hq = a->hq; p.hkv = a->hkv; p.tq = a->tq; p.d = a->d; p.nb = nb; p.bd = a->bd;
  p.k = a->k; p.nrep = a->hq / a->hkv; p.n_heavy = a->n_heavy;
  p.R = pl.R; p.tile = pl.tile; p.n_rg = pl.n_rg; p.n_ct = pl.n_ct; p.n_tt = pl.n_tt;
  p.tpu = pl.tpu; p.tc = a->tc; p.ttail = a->ttail; p.total_tiles = pl.total_tiles;
  p.n_units = pl.n_units; p.grid = pl.grid; p.stages = pl.stages;
  p.stage_shift = pl.stages == 4 ? 2 : (pl.stages == 2 ? 1 : 0); p.max_cov = pl.max_cov;
  p.w_unit = pl.w_unit;
  p.q = a->q; p.qdt = a->q_dtype; p.q_sb = a->q_sb; p.q_sh = a->q_sh; p.q_st = a->q_st;
  p.scale = a->scale;
  p.perm = a->perm; p.rot_k = a->rot_k; p.cents = a->centroids; p.heavy = a->heavy;
  p.idx = a->idx; p.idx_ps = a->idx_pair_stride;
  p.kheavy = a->kheavy; p.kh_ps = a->kheavy_pair_stride;
  p.vfmt = a->vfmt; p.v_ps = a->v_pair_stride; p.vq = a->vq; p.vq_ps = a->vq_pair_stride;
  p.vdec = a->vfmt == SS_V_F16 ? 0
           : a->vfmt == SS_V_VQ ? 2
           : (a->d == 128 && a->v_bits == 2 && a->v_group == 32 && a->v_scale_dtype == SS_F16 &&
              !a->v_zeros) ? 4
           : (a->d == 128 && a->v_bits == 2 && a->v_group % 16 == 0) ? 1 : 3;
  p.v_gshift = -1;
  for (int sh = 0; sh < 12; ++sh)
    if (a->v_group == (1 << sh)) p.v_gshift = sh;
  p.v_bits = a->v_bits; p.v_group = a->v_group; p.v_words = pl.v_words; p.v_groups = pl.v_groups;
  p.vs = a->v_scales; p.vs_dt = a->v_scale_dtype; p.vs_ps = a->vs_pair_stride;
  p.vz = a->v_zeros; p.vz_ps = a->vz_pair_stride;
  for (int i = 0; i < 16; ++i) p.levels[i] = a->v_levels[i];
  p.v_rot = a->v_rot;
  p.vidx = a->v_idx; p.vi_ps = a->vi_pair_stride; p.vcents = a->v_cents;
  p.v_bd = a->v_bd; p.v_k = a->v_k; p.v_nb = a->v_bd > 0 ? a->d / a->v_bd : 0;
  p.v_tile_bytes = pl.v_tile_bytes; p.off_vtab = pl.off_vtab;
  p.k_tail = a->k_tail; p.v_tail = a->v_tail; p.tail_ps = a->tail_pair_stride;
  p.causal = a->causal; p.mask = a->mask; p.mask_stride = a->mask_stride;
  p.mask_mode = a->mask_mode;
  p.out = a->out; p.odt = a->out_dtype; p.o_sb = a->o_sb; p.o_sh = a->o_sh; p.o_st = a->o_st;
  p.part_out = part_out;
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  p.err = reinterpret_cast<int*>(ws);
  p.sink = error_sink();
  p.wait_ns = a->wait_limit_ns > 0 ? static_cast<uint64_t>(a->wait_limit_ns) : kWaitLimitNs;
  p.skip_tile = a->test_skip_tile > 0 ? a->test_skip_tile - 1 : -1;
  p.counters = reinterpret_cast<int*>(ws + pl.off_counters);
  p.slots = reinterpret_cast<float*>(ws + pl.off_slots);
  p.lut_g = reinterpret_cast<float*>(ws + pl.off_lut_g);
  p.lut_unit_bytes = static_cast<uint32_t>(pl.lut_unit_bytes);
  p.lut_groups = static_cast<int>((pl.n_units + kLutUnits - 1) / kLutUnits);
  p.app_rows = 0;
  p.app_groups = 0;
  if (a->app_keys) {
    const int64_t rows = (int64_t)a->b * a->hkv * a->app_rows;
    SS_REQUIRE(a->app_values && a->app_rows >= 1 && a->app_rows <= a->tc,
               "ss_decode_attn: bad fused append (app_values / app_rows)");
    SS_REQUIRE(a->app_dtype >= SS_F32 && a->app_dtype <= SS_BF16, "ss_decode_attn: bad app_dtype");
    if (!(a->vfmt == SS_V_F16 && a->ttail == 0 && a->rot_k == nullptr &&
          (a->bd == 4 || a->bd == 8) && rows <= 4096))
      return fail(SS_ERR_UNSUPPORTED, "ss_decode_attn: fused append needs fp16 values, no fp16 "
                                      "tail, a permutation codec with 4- or 8-dim blocks and "
                                      "<= 4096 appended rows");
    p.app_k = a->app_keys; p.app_v = a->app_values; p.app_dt = a->app_dtype;
    p.app_kps = a->app_key_pair_stride; p.app_krs = a->app_key_row_stride;
    p.app_vps = a->app_value_pair_stride; p.app_vrs = a->app_value_row_stride;
    p.app_rows = a->app_rows;
    p.app_groups = static_cast<int>((rows + kAppRows - 1) / kAppRows);
    p.v_w = const_cast<uint16_t*>(reinterpret_cast<const uint16_t*>(a->v));
    count_dispatch("ss_cache_append (fused into ss_decode_attn)");
  }
  p.stage_bytes = pl.stage_bytes; p.off_idx = pl.off_idx; p.off_aux = pl.off_aux;
  p.off_vdq = pl.off_vdq; p.off_lut = pl.off_lut; p.off_p = pl.off_p; p.off_misc = pl.off_misc;
  p.off_plo = pl.off_plo;
  p.off_stage = 0;
  count_dispatch(name ? name : (part_out ? "ss_decode_attn_partial" : "ss_decode_attn"));
#define SS_DISPATCH(RV, DV) \
  if (pl.R == RV && a->d == DV) return launch_decode<RV, DV>(p, mv, mvt, pl.smem, pl.cw, st);
  SS_DISPATCH(1, 128) SS_DISPATCH(2, 128) SS_DISPATCH(4, 128) SS_DISPATCH(8, 128)
  SS_DISPATCH(1, 64) SS_DISPATCH(2, 64) SS_DISPATCH(4, 64) SS_DISPATCH(8, 64)
#undef SS_DISPATCH
  return fail(SS_ERR_UNSUPPORTED, "ss_decode_attn: no kernel for this configuration");
}

}  // namespace
}  // namespace ss

using namespace ss;

extern "C" {

size_t ss_decode_workspace_size(const ss_decode_args* a) {
  Plan pl;
  if (make_plan(a, pl) != SS_OK) return 0;
  return pl.ws_bytes;
}

int ss_decode_attn(const ss_decode_args* a, void* stream) { return run_decode(a, nullptr, stream); }

int ss_decode_attn_partial(const ss_decode_args* a, float* part_out, void* stream) {
  SS_REQUIRE(part_out, "ss_decode_attn_partial: null part_out");
  return run_decode(a, part_out, stream);
}

int ss_decode_check(void* workspace, void* stream) {
  SS_REQUIRE(workspace, "ss_decode_check: null workspace");
  int h = 0;
  cudaStream_t st = as_stream(stream);
  if (cudaMemcpyAsync(&h, workspace, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return check_launch("ss_decode_check");
  if (h != 0) {
    cudaMemsetAsync(workspace, 0, sizeof(int), st);
    cudaStreamSynchronize(st);
    return fail(SS_ERR_TIMEOUT, "ss_decode_attn: a device-side wait timed out (code " +
                                    std::to_string(h) + ")");
  }
  return SS_OK;
}

int ss_lse_merge(const float* parts, int n_parts, int64_t rows, int d, const float* v_rot,
                 void* out, int out_dtype, int64_t out_stride, void* stream) {
  SS_REQUIRE(parts && out, "ss_lse_merge: null pointer");
  SS_REQUIRE(n_parts >= 1 && n_parts <= 64 && d > 0 && d <= 512, "ss_lse_merge: bad sizes");
  count_dispatch("ss_lse_merge");
  if (rows <= 0) return SS_OK;
  lse_merge_kernel<<<static_cast<unsigned>(rows), 128, 0, as_stream(stream)>>>(
      parts, n_parts, rows, d, v_rot, out, out_dtype, out_stride);
  return check_launch("ss_lse_merge");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode attention without any allocation by the caller.
//
// Some callers cannot allocate device memory at the point where they run
// attention: allocator-less runtimes, code running inside another
// framework's memory pool that forbids extra cudaMalloc traffic, or hosts
// that only hand over pre-registered input/output buffers. For them the
// decode workspace (error word, per-unit arrival counters, cross-CTA partial
// rows) lives in this fixed device array instead of a caller buffer.
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per device
static __device__ __align__(256) uint8_t g_decode_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {nullptr};

// Device address of g_decode_scratch on the current device (looked up once).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(SS_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(SS_ERR_UNSUPPORTED, "ss_decode_attn_noalloc: device index >= 64");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(SS_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return SS_OK;
}
}  // namespace

extern "C" int ss_decode_attn_noalloc(const ss_decode_args* a, void* stream) {
  SS_REQUIRE(a, "ss_decode_attn_noalloc: null args");
  Plan pl;
  int rc = make_plan(a, pl);
  if (rc != SS_OK) return rc;
  if (pl.ws_bytes > kNoAllocScratchBytes)
    return fail(SS_ERR_WORKSPACE,
                "ss_decode_attn_noalloc: this problem needs " + std::to_string(pl.ws_bytes) +
                    " bytes of decode scratch, more than the fixed " +
                    std::to_string(kNoAllocScratchBytes) +
                    " bytes; use ss_decode_attn with a caller workspace");
  void* scratch = nullptr;
  rc = scratch_address(&scratch);
  if (rc != SS_OK) return rc;
  // the arrival counters must start at zero (the array keeps the previous
  // call's contents); the error word before them stays sticky until
  // ss_decode_noalloc_check reads it
  cudaError_t e = cudaMemsetAsync(static_cast<uint8_t*>(scratch) + pl.off_counters, 0,
                                  pl.off_slots - pl.off_counters, as_stream(stream));
  if (e != cudaSuccess)
    return fail(SS_ERR_CUDA, std::string("ss_decode_attn_noalloc: memset: ") + cudaGetErrorString(e));
  ss_decode_args b = *a;
  b.workspace = scratch;
  b.workspace_bytes = kNoAllocScratchBytes;
  return run_decode(&b, nullptr, stream, "ss_decode_attn_noalloc");
}

extern "C" int ss_decode_noalloc_check(void* stream) {
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != SS_OK) return rc;
  return ss_decode_check(scratch, stream);
}
