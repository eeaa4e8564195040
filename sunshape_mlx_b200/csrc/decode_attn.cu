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
#include <cfloat>

#include "common.cuh"

namespace ss {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;
constexpr int kMaxStages = 8;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per barrier wait
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeParams {
  // shapes
  int b, hq, hkv, tq, d, nb, bd, k, nrep, n_heavy;
  int R, tile, n_rg, n_ct, n_tt, tpu;
  int64_t tc, ttail, total_tiles, n_units;
  int grid, stages, max_cov;
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
  const void* vs;
  int vs_dt;
  int64_t vs_ps;
  const float* vz;
  int64_t vz_ps;
  float levels[16];
  const float* v_rot;
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
  int* counters;
  float* slots;
  // shared-memory carve-up (bytes from the 1024-aligned base)
  uint32_t off_stage, stage_bytes, off_idx, off_aux, off_vdq, off_lut, off_p, off_misc;
};

__device__ __forceinline__ int64_t cta_of(int64_t tile, int64_t total, int grid) {
  return ((tile + 1) * grid - 1) / total;
}
__device__ __forceinline__ int64_t range_start(int64_t i, int64_t total, int grid) {
  return i * total / grid;
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
  float o[8][128];      // finalisation staging
  float mrow[8], lrow[8];
  float levels[16];
  int heavy_pos[32];
  uint8_t is_heavy[128];
  int is_last;
  int abort;
};

template <int R, int D>
__global__ void __launch_bounds__(kThreads, 1) decode_attn_kernel(
    const __grid_constant__ DecodeParams p, const __grid_constant__ CUtensorMap map_v,
    const __grid_constant__ CUtensorMap map_vt) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full_bar[kMaxStages], empty_bar[kMaxStages];

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int TILE = p.tile;
  const int wpt = TILE / 16;                   // warps sharing one tile (16 tokens each)
  Misc& ms = *reinterpret_cast<Misc*>(smem + p.off_misc);
  float* lut = reinterpret_cast<float*>(smem + p.off_lut);

  const int64_t cta = blockIdx.x;
  const int64_t t_begin = range_start(cta, p.total_tiles, p.grid);
  const int64_t t_end = range_start(cta + 1, p.total_tiles, p.grid);

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], wpt);
    }
    ms.abort = 0;
    int hp = 0;
    for (int b = 0; b < p.nb; ++b) {
      const bool hv = p.heavy && p.heavy[b];
      ms.is_heavy[b] = hv ? 1 : 0;
      if (hv && hp < 32) ms.heavy_pos[hp++] = b;
    }
    for (int i = 0; i < 16; ++i) ms.levels[i] = p.levels[i];
    fence_mbar_init();
  }
  __syncthreads();

  // ====================================================== producer warp
  if (warp == kConsumerWarps) {
    if (lane == 0) {
      if (p.vfmt == SS_V_F16 && p.n_ct > 0) prefetch_tmap(&map_v);
      if (p.n_tt > 0 && p.vfmt == SS_V_F16) prefetch_tmap(&map_vt);
      int it = 0;
      for (int64_t tau = t_begin; tau < t_end; ++tau, ++it) {
        const int s = it % p.stages;
        if (it >= p.stages) {
          if (ms.abort || !mbar_wait_bounded(&empty_bar[s], ((it / p.stages) - 1) & 1,
                                             kWaitLimitNs)) {
            ms.abort = 1;
            atomicOr(p.err, 1);
            break;
          }
        }
        const int64_t u = tau / p.tpu;
        const int lt = static_cast<int>(tau - u * p.tpu);
        const int64_t pair = u / p.n_rg;
        uint8_t* st = smem + (size_t)s * p.stage_bytes;
        if (lt < p.n_ct) {
          const int64_t t0 = (int64_t)lt * TILE;
          uint32_t bytes = TILE * p.nb;
          if (p.vfmt == SS_V_F16) bytes += TILE * D * 2;
          else {
            bytes += TILE * p.v_words * 4 + TILE * p.v_groups * (p.vs_dt == SS_F32 ? 4 : 2);
            if (p.vz) bytes += TILE * p.v_groups * 4;
          }
          if (p.n_heavy) bytes += TILE * p.n_heavy * p.bd * 2;
          mbar_arrive_expect_tx(&full_bar[s], bytes);
          bulk_g2s(st + p.off_idx, p.idx + pair * p.idx_ps + t0 * p.nb, TILE * p.nb,
                   &full_bar[s]);
          uint8_t* aux = st + p.off_aux;
          if (p.vfmt == SS_V_F16) {
            for (int bx = 0; bx < D / 64; ++bx)
              tma_load_3d(st + bx * TILE * 128, &map_v, bx * 64, static_cast<int32_t>(t0),
                          static_cast<int32_t>(pair), &full_bar[s]);
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
      // Drain: make sure no copy issued by this CTA is still in flight.
      const int issued = it;
      for (int j = issued - p.stages; j < issued; ++j) {
        if (j < 0) continue;
        const int s = j % p.stages;
        if (!mbar_wait_bounded(&full_bar[s], (j / p.stages) & 1, kWaitLimitNs)) {
          atomicOr(p.err, 2);
          break;
        }
      }
    }
    return;
  }

  // ====================================================== consumer warps
  // Warp w owns 16-token slice (w % wpt) of every tile of tile group (w / wpt);
  // two lanes per token, each summing half of the blocks.
  constexpr int MT = D / 16;                   // 16-dim MMA tiles of the output
  const int tgroups = kConsumerWarps / wpt;
  const int wgroup = warp / wpt, slice = warp % wpt;
  const int ltok = lane >> 1, part = lane & 1;
  const int tok = slice * 16 + ltok;           // token within the tile
  const int nbp = p.nb / 2;
  const int ctid = tid;                        // 0..255
  const int64_t q_off = p.tc + p.ttail - p.tq;
  __half* Pw = reinterpret_cast<__half*>(smem + p.off_p) + warp * 16 * 8;  // [16][8]
  uint8_t* vdq_w = smem + p.off_vdq + warp * (16 * D * 2);
  const uint32_t pw_addr = smem_u32(Pw) + (lane & 15) * 16;
  const int mi = lane >> 3, mj = lane & 7;
  const int kk_off = (mi >= 2 ? 8 : 0) + mj;   // ldmatrix row (token) of this lane
  const int dim_off = (mi & 1) ? 8 : 0;
  const int rows_valid = p.nrep * p.tq;

  int64_t tau = t_begin;
  while (tau < t_end) {
    const int64_t u = tau / p.tpu;
    const int64_t u_end = min(t_end, (u + 1) * p.tpu);
    const int64_t pair = u / p.n_rg;
    const int rg = static_cast<int>(u - pair * p.n_rg);
    const int bb = static_cast<int>(pair / p.hkv), hh = static_cast<int>(pair % p.hkv);

    // ---------------------------------------------- build the unit's LUT
    named_bar_sync(1, kConsumers);  // previous unit finalised, LUT region free
    {
      const float sc = round_to(p.scale, p.qdt);
      for (int e = ctid; e < R * p.d; e += kConsumers) {
        const int r = e / p.d, j = e - r * p.d;
        const int rr = rg * R + r;
        float v = 0.f;
        if (rr < rows_valid) {
          const int rep = rr / p.tq, tqi = rr - rep * p.tq;
          const int qh = hh * p.nrep + rep;
          const float x = load_as_f32(p.q, p.qdt, bb * p.q_sb + qh * p.q_sh + tqi * p.q_st + j);
          v = round_to(x * sc, p.qdt);
        }
        ms.qo[r][j] = v;
      }
      named_bar_sync(1, kConsumers);
      for (int e = ctid; e < R * p.d; e += kConsumers) {
        const int r = e / p.d, j = e - r * p.d;
        float v;
        if (p.rot_k) {
          float a = 0.f;
          for (int i = 0; i < p.d; ++i) a = fmaf(ms.qo[r][i], p.rot_k[j * p.d + i], a);
          v = a;
        } else {
          v = ms.qo[r][p.perm ? p.perm[j] : j];
        }
        ms.qc[r][j] = v;
      }
      named_bar_sync(1, kConsumers);
      for (int e = ctid; e < p.nb * p.k; e += kConsumers) {
        const int b = e / p.k;
        const float* c = p.cents + (size_t)e * p.bd;
        // Heavy blocks are scored exactly from their fp16 values when the
        // cache stores them (n_heavy > 0); their table entries are zero then.
        const bool zero = p.n_heavy > 0 && ms.is_heavy[b];
        float cv[16];
        for (int j = 0; j < p.bd; ++j) cv[j] = zero ? 0.f : __ldg(c + j);
        float* dst = lut + (size_t)e * R;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float a = 0.f;
          for (int j = 0; j < p.bd; ++j) a = fmaf(ms.qc[r][b * p.bd + j], cv[j], a);
          dst[r] = a;
        }
      }
      named_bar_sync(1, kConsumers);
    }

    // ---------------------------------------------- this warp's slices of the unit
    float m_w[R], l_l[R];
    float acc[MT][4];
#pragma unroll
    for (int r = 0; r < R; ++r) { m_w[r] = -INFINITY; l_l[r] = 0.f; }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;

    for (int64_t t2 = tau; t2 < u_end; ++t2) {
      const int it = static_cast<int>(t2 - t_begin);
      if (it % tgroups != wgroup) continue;
      const int lt = static_cast<int>(t2 - u * p.tpu);
      const int s = it % p.stages;
      if (!ms.abort && !mbar_wait_bounded(&full_bar[s], (it / p.stages) & 1, kWaitLimitNs)) {
        ms.abort = 1;
        atomicOr(p.err, 4);
      }
      const bool aborted = ms.abort != 0;
      uint8_t* st = smem + (size_t)s * p.stage_bytes;
      const bool compressed = lt < p.n_ct;
      const int64_t t0 = compressed ? (int64_t)lt * TILE : (int64_t)(lt - p.n_ct) * TILE;
      const int64_t len = compressed ? p.tc : p.ttail;
      const int64_t t = t0 + tok;
      const bool tvalid = t < len && !aborted;
      const int64_t tg = compressed ? t : p.tc + t;

      // 1. scores of this lane's token (half of the blocks)
      float sc[R];
#pragma unroll
      for (int r = 0; r < R; ++r) sc[r] = 0.f;
      if (tvalid) {
        if (compressed) {
          const uint8_t* irow = st + p.off_idx + tok * p.nb + part * nbp;
          for (int j0 = 0; j0 < nbp; j0 += 8) {
            const uint2 raw = *reinterpret_cast<const uint2*>(irow + j0);
            const uint32_t w2[2] = {raw.x, raw.y};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              if (j0 + j >= nbp) break;
              const int b = part * nbp + j0 + j;
              const uint32_t c = (w2[j >> 2] >> ((j & 3) * 8)) & 0xffu;
              const float* e = lut + ((size_t)b * p.k + c) * R;
              if constexpr (R == 4) {
                const float4 v = *reinterpret_cast<const float4*>(e);
                sc[0] += v.x; sc[1] += v.y; sc[2] += v.z; sc[3] += v.w;
              } else if constexpr (R == 8) {
                const float4 v0 = *reinterpret_cast<const float4*>(e);
                const float4 v1 = *reinterpret_cast<const float4*>(e + 4);
                sc[0] += v0.x; sc[1] += v0.y; sc[2] += v0.z; sc[3] += v0.w;
                sc[4] += v1.x; sc[5] += v1.y; sc[6] += v1.z; sc[7] += v1.w;
              } else {
#pragma unroll
                for (int r = 0; r < R; ++r) sc[r] += e[r];
              }
            }
          }
          if (p.n_heavy) {
            int off = p.off_aux;
            if (p.vfmt != SS_V_F16) {
              off += TILE * p.v_words * 4 + TILE * p.v_groups * (p.vs_dt == SS_F32 ? 4 : 2);
              if (p.vz) off += TILE * p.v_groups * 4;
            }
            const uint16_t* hrow =
                reinterpret_cast<const uint16_t*>(st + off) + (size_t)tok * p.n_heavy * p.bd;
            for (int hj = part; hj < p.n_heavy; hj += 2) {
              const int b = ms.heavy_pos[hj];
              for (int j = 0; j < p.bd; ++j) {
                const float kv = h2f(hrow[hj * p.bd + j]);
#pragma unroll
                for (int r = 0; r < R; ++r) sc[r] = fmaf(ms.qc[r][b * p.bd + j], kv, sc[r]);
              }
            }
          }
        } else {
          const uint16_t* krow = p.k_tail + pair * p.tail_ps + t * D;
          constexpr int per = D / 2;
          for (int j0 = part * per; j0 < (part + 1) * per; j0 += 8) {
            const uint4 raw = *reinterpret_cast<const uint4*>(krow + j0);
            const uint16_t* hv = reinterpret_cast<const uint16_t*>(&raw);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float kv = h2f(hv[j]);
#pragma unroll
              for (int r = 0; r < R; ++r) sc[r] = fmaf(ms.qo[r][j0 + j], kv, sc[r]);
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < R; ++r) sc[r] += __shfl_xor_sync(0xffffffffu, sc[r], 1);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int rr = rg * R + r;
        bool ok = tvalid && rr < rows_valid;
        const int tqi = rr % p.tq;
        if (ok && p.causal && tg > q_off + tqi) ok = false;
        if (ok && p.mask) {
          const float mv = p.mask[tqi * p.mask_stride + tg];
          if (p.mask_mode == 0) sc[r] += mv;
          else if (mv == 0.f) sc[r] = -FLT_MAX;
        }
        if (!ok) sc[r] = -INFINITY;
      }

      // 2. online softmax over this warp's slice
      float alpha[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float mx = sc[r];
#pragma unroll
        for (int o = 2; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float mn = fmaxf(m_w[r], mx);
        alpha[r] = (mn == -INFINITY) ? 1.f : exp2f((m_w[r] - mn) * kLog2e);
        const float e = (sc[r] == -INFINITY) ? 0.f : exp2f((sc[r] - mn) * kLog2e);
        const __half h = __float2half_rn(e);
        if (part == 0) {
          Pw[ltok * 8 + r] = h;
          l_l[r] = l_l[r] * alpha[r] + __half2float(h);
        } else {
          l_l[r] *= alpha[r];
        }
        m_w[r] = mn;
      }
      if (part == 0) {
#pragma unroll
        for (int r = R; r < 8; ++r) Pw[ltok * 8 + r] = __float2half_rn(0.f);
      }

      // quantized values (or the quantized path's tail) -> this warp's fp16 slice
      uint32_t vbase;
      int vrows, vtok;
      if (p.vfmt == SS_V_F16) {
        vbase = smem_u32(st);
        vrows = TILE;
        vtok = slice * 16;
      } else {
        vbase = smem_u32(vdq_w);
        vrows = 16;
        vtok = 0;
        if (compressed) {
          const uint32_t* words = reinterpret_cast<const uint32_t*>(st + p.off_aux);
          const uint8_t* sp = st + p.off_aux + TILE * p.v_words * 4;
          const float* zp = p.vz ? reinterpret_cast<const float*>(
                                       sp + TILE * p.v_groups * (p.vs_dt == SS_F32 ? 4 : 2))
                                 : nullptr;
          const int vpw = p.v_bits == 3 ? 10 : 32 / p.v_bits;
          const uint32_t msk = (1u << p.v_bits) - 1u;
          for (int e = lane; e < 16 * (D / 8); e += 32) {
            const int tk = e / (D / 8), ch = e - tk * (D / 8);
            const int tt = slice * 16 + tk;
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
            const int64_t tt = t0 + slice * 16 + tk;
            uint4 pk = make_uint4(0, 0, 0, 0);
            if (tt < len)
              pk = *reinterpret_cast<const uint4*>(p.v_tail + pair * p.tail_ps + tt * D + ch * 8);
            *reinterpret_cast<uint4*>(vdq_w + vtile_addr(0, 16, tk, ch * 8)) = pk;
          }
        }
      }
      __syncwarp();

      // 3. P.V: O^T[dims][rows] += V^T[dims][16 tokens] . P[16 tokens][rows]
      {
        const int n0 = 2 * (lane & 3);
        float a0 = 1.f, a1 = 1.f;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          if (r == n0) a0 = alpha[r];
          if (r == n0 + 1) a1 = alpha[r];
        }
        uint32_t b0, b1;
        ldsm_x2_trans(pw_addr, b0, b1);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          acc[mt][0] *= a0; acc[mt][1] *= a1; acc[mt][2] *= a0; acc[mt][3] *= a1;
          uint32_t x0, x1, x2, x3;
          ldsm_x4_trans(vtile_addr(vbase, vrows, vtok + kk_off, mt * 16 + dim_off), x0, x1, x2, x3);
          mma_16816(acc[mt], x0, x1, x2, x3, b0, b1);
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
    named_bar_sync(1, kConsumers);  // every warp is done with the LUT: reuse it as scratch
    float* wo = lut;                                  // [8][R][D]
    float* wm = lut + kConsumerWarps * R * D;         // [8][R]
    float* wl = wm + kConsumerWarps * R;              // [8][R]
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
    named_bar_sync(1, kConsumers);
    for (int e = ctid; e < R * D; e += kConsumers) {
      const int r = e / D, j = e - r * D;
      float mstar = -INFINITY;
      for (int w = 0; w < kConsumerWarps; ++w) mstar = fmaxf(mstar, wm[w * R + r]);
      float O = 0.f, L = 0.f;
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float mg = wm[w * R + r];
        const float wt = (mg == -INFINITY) ? 0.f : exp2f((mg - mstar) * kLog2e);
        O = fmaf(wo[(w * R + r) * D + j], wt, O);
        L = fmaf(wl[w * R + r], wt, L);
      }
      ms.o[r][j] = O;
      if (j == 0) { ms.mrow[r] = mstar; ms.lrow[r] = L; }
    }
    named_bar_sync(1, kConsumers);

    // ---------------------------------------------- unit finalisation
    const int64_t first = cta_of(u * p.tpu, p.total_tiles, p.grid);
    const int64_t last = cta_of((u + 1) * p.tpu - 1, p.total_tiles, p.grid);
    const int ncov = static_cast<int>(last - first + 1);
    const int row_floats = D + 2;
    bool do_final = true;
    if (ncov > 1) {
      float* slot = p.slots + ((size_t)u * p.max_cov + (cta - first)) * R * row_floats;
      for (int e = ctid; e < R * row_floats; e += kConsumers) {
        const int r = e / row_floats, j = e - r * row_floats;
        slot[e] = j < D ? ms.o[r][j] : (j == D ? ms.mrow[r] : ms.lrow[r]);
      }
      __threadfence();
      named_bar_sync(1, kConsumers);
      if (ctid == 0) {
        const int prev = atomicAdd(p.counters + u, 1);
        if (prev == ncov - 1) {
          ms.is_last = 1;
          p.counters[u] = 0;  // leave the counter ready for the next launch
        }
      }
      named_bar_sync(1, kConsumers);
      do_final = ms.is_last != 0;
      if (do_final) {
        __threadfence();
        const float* base = p.slots + (size_t)u * p.max_cov * R * row_floats;
        for (int e = ctid; e < R * D; e += kConsumers) {
          const int r = e / D, j = e - r * D;
          float mstar = -INFINITY;
          for (int g = 0; g < ncov; ++g)
            mstar = fmaxf(mstar, __ldcg(base + ((size_t)g * R + r) * row_floats + D));
          float O = 0.f, L = 0.f;
          for (int g = 0; g < ncov; ++g) {
            const float* row = base + ((size_t)g * R + r) * row_floats;
            const float mg = __ldcg(row + D);
            const float w = (mg == -INFINITY) ? 0.f : exp2f((mg - mstar) * kLog2e);
            O = fmaf(__ldcg(row + j), w, O);
            L = fmaf(__ldcg(row + D + 1), w, L);
          }
          ms.o[r][j] = O;
          if (j == 0) { ms.mrow[r] = mstar; ms.lrow[r] = L; }
        }
        named_bar_sync(1, kConsumers);
      }
    }
    if (do_final) {
      for (int e = ctid; e < R * D; e += kConsumers) {
        const int r = e / D, j = e - r * D;
        const int rr = rg * R + r;
        if (rr >= rows_valid) continue;
        const int rep = rr / p.tq, tqi = rr - rep * p.tq;
        const int qh = hh * p.nrep + rep;
        if (p.part_out) {
          float* row = p.part_out + (((int64_t)bb * p.hq + qh) * p.tq + tqi) * (D + 2);
          row[j] = ms.o[r][j];
          if (j == 0) { row[D] = ms.mrow[r]; row[D + 1] = ms.lrow[r]; }
        } else {
          const float inv = ms.lrow[r] > 0.f ? 1.f / ms.lrow[r] : 0.f;
          float v;
          if (p.v_rot) {
            float a = 0.f;
            for (int i = 0; i < D; ++i) a = fmaf(ms.o[r][i], __ldg(p.v_rot + i * D + j), a);
            v = a * inv;
          } else {
            v = ms.o[r][j] * inv;
          }
          store_from_f32(p.out, p.odt, bb * p.o_sb + qh * p.o_sh + tqi * p.o_st + j, v);
        }
      }
    }
    tau = u_end;
  }
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
  int R, tile, n_rg, n_ct, n_tt, tpu, grid, stages, max_cov, v_words, v_groups;
  int64_t total_tiles, n_units;
  uint32_t stage_bytes, off_idx, off_aux, off_vdq, off_lut, off_p, off_misc;
  size_t smem;
  size_t ws_bytes, off_counters, off_slots;
};

constexpr size_t kSmemBudget = 226 * 1024;  // leaves room for static barriers

int make_plan(const ss_decode_args* a, Plan& pl) {
  SS_REQUIRE(a, "ss_decode_attn: null args");
  SS_REQUIRE(a->d == 64 || a->d == 128, "ss_decode_attn: head_dim must be 64 or 128");
  SS_REQUIRE(a->bd > 0 && a->bd <= 16 && a->d % a->bd == 0, "ss_decode_attn: bad block_dim");
  SS_REQUIRE(a->k >= 1 && a->k <= 256, "ss_decode_attn: k must be in [1, 256]");
  SS_REQUIRE(a->hkv > 0 && a->hq % a->hkv == 0, "ss_decode_attn: hq must be a multiple of hkv");
  SS_REQUIRE(a->b >= 0 && a->tq >= 1 && a->tc >= 0 && a->ttail >= 0,
             "ss_decode_attn: bad batch / lengths");
  SS_REQUIRE(a->vfmt == SS_V_F16 || a->vfmt == SS_V_QUANT, "ss_decode_attn: bad vfmt");
  SS_REQUIRE(a->n_heavy >= 0 && a->n_heavy <= 32, "ss_decode_attn: n_heavy must be <= 32");
  const int nb = a->d / a->bd;
  const int nrep = a->hq / a->hkv;
  const int rows = nrep * a->tq;
  int R = rows >= 5 ? 8 : (rows >= 3 ? 4 : (rows == 2 ? 2 : 1));
  while (R > 1 && (size_t)nb * a->k * R * 4 > 128 * 1024) R >>= 1;
  pl.R = R;
  pl.tile = R <= 4 ? 128 : 64;
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
  const int64_t per_cta = pl.total_tiles / pl.grid;
  pl.max_cov = static_cast<int>(pl.tpu / (per_cta > 0 ? per_cta : 1)) + 2;
  if (pl.max_cov > pl.grid) pl.max_cov = pl.grid;
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
  }
  aux += T * a->n_heavy * a->bd * 2;
  pl.stage_bytes = (pl.off_aux + aux + 1023) & ~1023u;
  size_t fixed = 0;
  // per-warp fp16 value slices (16 tokens) for the quantized path
  const size_t vdq = (a->vfmt == SS_V_QUANT) ? (size_t)kConsumerWarps * 16 * a->d * 2 : 0;
  // the LUT region doubles as the per-warp merge scratch at unit ends
  size_t lut = (size_t)nb * a->k * R * 4;
  const size_t scratch = (size_t)kConsumerWarps * R * (a->d + 2) * 4;
  if (lut < scratch) lut = scratch;
  const size_t pbytes = (size_t)kConsumerWarps * 16 * 16;
  fixed = vdq + ((lut + 127) & ~size_t(127)) + pbytes + ((sizeof(Misc) + 127) & ~size_t(127)) + 1024;
  if (fixed + 2 * (size_t)pl.stage_bytes > kSmemBudget)
    return fail(SS_ERR_UNSUPPORTED, "ss_decode_attn: configuration exceeds shared memory");
  int stages = static_cast<int>((kSmemBudget - fixed) / pl.stage_bytes);
  if (stages > 4) stages = 4;
  pl.stages = stages;
  size_t off = (size_t)stages * pl.stage_bytes;
  pl.off_vdq = static_cast<uint32_t>(off);
  off += vdq;
  pl.off_lut = static_cast<uint32_t>(off);
  off += (lut + 127) & ~size_t(127);
  pl.off_p = static_cast<uint32_t>(off);
  off += pbytes;
  pl.off_misc = static_cast<uint32_t>(off);
  off += (sizeof(Misc) + 127) & ~size_t(127);
  pl.smem = off + 1024;
  // workspace: [error word | counters | partial slots]
  pl.off_counters = 256;
  pl.off_slots = (pl.off_counters + (size_t)pl.n_units * 4 + 255) & ~size_t(255);
  pl.ws_bytes = pl.off_slots + (size_t)pl.n_units * pl.max_cov * R * (a->d + 2) * 4;
  return SS_OK;
}

template <int R, int D>
int launch_decode(const DecodeParams& p, const CUtensorMap& mv, const CUtensorMap& mvt,
                  size_t smem, cudaStream_t st) {
  auto kern = decode_attn_kernel<R, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess)
    return fail(SS_ERR_CUDA, std::string("ss_decode_attn: smem attribute: ") + cudaGetErrorString(e));
  kern<<<p.grid, kThreads, smem, st>>>(p, mv, mvt);
  return check_launch("ss_decode_attn");
}

int run_decode(const ss_decode_args* a, float* part_out, void* stream) {
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
  p.n_units = pl.n_units; p.grid = pl.grid; p.stages = pl.stages; p.max_cov = pl.max_cov;
  p.q = a->q; p.qdt = a->q_dtype; p.q_sb = a->q_sb; p.q_sh = a->q_sh; p.q_st = a->q_st;
  p.scale = a->scale;
  p.perm = a->perm; p.rot_k = a->rot_k; p.cents = a->centroids; p.heavy = a->heavy;
  p.idx = a->idx; p.idx_ps = a->idx_pair_stride;
  p.kheavy = a->kheavy; p.kh_ps = a->kheavy_pair_stride;
  p.vfmt = a->vfmt; p.v_ps = a->v_pair_stride; p.vq = a->vq; p.vq_ps = a->vq_pair_stride;
  p.v_bits = a->v_bits; p.v_group = a->v_group; p.v_words = pl.v_words; p.v_groups = pl.v_groups;
  p.vs = a->v_scales; p.vs_dt = a->v_scale_dtype; p.vs_ps = a->vs_pair_stride;
  p.vz = a->v_zeros; p.vz_ps = a->vz_pair_stride;
  for (int i = 0; i < 16; ++i) p.levels[i] = a->v_levels[i];
  p.v_rot = a->v_rot;
  p.k_tail = a->k_tail; p.v_tail = a->v_tail; p.tail_ps = a->tail_pair_stride;
  p.causal = a->causal; p.mask = a->mask; p.mask_stride = a->mask_stride;
  p.mask_mode = a->mask_mode;
  p.out = a->out; p.odt = a->out_dtype; p.o_sb = a->o_sb; p.o_sh = a->o_sh; p.o_st = a->o_st;
  p.part_out = part_out;
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  p.err = reinterpret_cast<int*>(ws);
  p.counters = reinterpret_cast<int*>(ws + pl.off_counters);
  p.slots = reinterpret_cast<float*>(ws + pl.off_slots);
  p.stage_bytes = pl.stage_bytes; p.off_idx = pl.off_idx; p.off_aux = pl.off_aux;
  p.off_vdq = pl.off_vdq; p.off_lut = pl.off_lut; p.off_p = pl.off_p; p.off_misc = pl.off_misc;
  p.off_stage = 0;
  count_dispatch(part_out ? "ss_decode_attn_partial" : "ss_decode_attn");
#define SS_DISPATCH(RV, DV) \
  if (pl.R == RV && a->d == DV) return launch_decode<RV, DV>(p, mv, mvt, pl.smem, st);
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
