// Value-codec kernels for the cache append path: grouped min-max and
// TurboQuant encoders, the scalar-quantized decoder, bit (un)packing and the
// scalar boundary quantizer.
//
// Layout: one warp per row; the row is staged as float32 in shared memory,
// codes are computed per channel and packed word by word with the reference's
// bit order (element i of a word at bits [i*bits, (i+1)*bits), 3-bit rows
// zero-padded to a multiple of 10, kernels.py:1102-1137).
#include "common.cuh"

namespace ss {
namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kMaxD = 512;

__device__ __forceinline__ int vals_per_word(int bits) { return bits == 3 ? 10 : 32 / bits; }

__device__ __forceinline__ int packed_words(int d, int bits) {
  return bits == 3 ? (d + 9) / 10 : d / (32 / bits);
}

// Packs codes[0..d) (uint8 in shared memory) into the row's words.
__device__ __forceinline__ void pack_row(const uint8_t* codes, int d, int bits, uint32_t* dst,
                                         int lane) {
  const int vpw = vals_per_word(bits);
  const int nw = packed_words(d, bits);
  const uint32_t m = (1u << bits) - 1u;
  for (int w = lane; w < nw; w += 32) {
    uint32_t word = 0;
    for (int i = 0; i < vpw; ++i) {
      const int c = w * vpw + i;
      if (c < d) word |= (static_cast<uint32_t>(codes[c]) & m) << (i * bits);
    }
    dst[w] = word;
  }
}

__device__ __forceinline__ float warp_min(float v) {
  for (int o = 16; o; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

struct RowAddr {
  int64_t n_groups, rpg;
  __device__ __forceinline__ void split(int64_t r, int64_t& g, int64_t& t) const {
    g = r / rpg;
    t = r - g * rpg;
  }
};

// ------------------------------------------------------------- grouped
__global__ void __launch_bounds__(kWarpsPerCta * 32)
    encode_grouped_kernel(const void* v, int vdt, RowAddr ra, int64_t vgs, int64_t vrs, int d,
                          int bits, int gs, uint32_t* packed, int64_t pgs, int64_t prs,
                          float* scales, float* zeros, int64_t sgs, int64_t srs) {
  __shared__ float s_v[kWarpsPerCta][kMaxD];
  __shared__ uint8_t s_code[kWarpsPerCta][kMaxD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_rows = ra.n_groups * ra.rpg;
  const int maxq = (1 << bits) - 1;
  const int ng = d / gs;
  for (int64_t r = (int64_t)blockIdx.x * kWarpsPerCta + warp; r < n_rows;
       r += (int64_t)gridDim.x * kWarpsPerCta) {
    int64_t g, t;
    ra.split(r, g, t);
    const int64_t vo = g * vgs + t * vrs;
    for (int c = lane; c < d; c += 32) s_v[warp][c] = load_as_f32(v, vdt, vo + c);
    __syncwarp();
    for (int gi = 0; gi < ng; ++gi) {
      float lo = INFINITY, hi = -INFINITY;
      for (int c = gi * gs + lane; c < (gi + 1) * gs; c += 32) {
        lo = fminf(lo, s_v[warp][c]);
        hi = fmaxf(hi, s_v[warp][c]);
      }
      lo = warp_min(lo);
      hi = warp_max(hi);
      float sc = __fdiv_rn(__fsub_rn(hi, lo), static_cast<float>(maxq));
      if (sc < 1e-8f) sc = 1e-8f;
      for (int c = gi * gs + lane; c < (gi + 1) * gs; c += 32) {
        float qv = rintf(__fdiv_rn(__fsub_rn(s_v[warp][c], lo), sc));
        qv = fminf(fmaxf(qv, 0.f), static_cast<float>(maxq));
        s_code[warp][c] = static_cast<uint8_t>(qv);
      }
      if (lane == 0) {
        scales[g * sgs + t * srs + gi] = sc;
        zeros[g * sgs + t * srs + gi] = lo;
      }
    }
    __syncwarp();
    pack_row(s_code[warp], d, bits, packed + g * pgs + t * prs, lane);
    __syncwarp();
  }
}

// Grouped min-max for fp16 rows of 128 values, 2- or 4-bit: a half-warp per row
// (lane = one 16-byte chunk of 8 values), group min / max by shuffles among
// the lanes of a group, the same fp32 arithmetic as the general kernel, and
// codes packed straight into words (4-bit: one word per lane; 2-bit: lane
// pairs). gs = group size (a multiple of 8 dividing 128).
template <int BITS>
__global__ void __launch_bounds__(256) encode_grouped_f16_kernel(
    const __half* v, RowAddr ra, int64_t vgs, int64_t vrs, int gs, uint32_t* packed,
    int64_t pgs, int64_t prs, float* scales, float* zeros, int64_t sgs, int64_t srs) {
  constexpr int maxq = (1 << BITS) - 1;
  const int lane = threadIdx.x & 31, half = lane >> 4, c = lane & 15;
  const int lpg = gs >> 3;  // lanes per group
  const int64_t n_rows = ra.n_groups * ra.rpg;
  const int64_t step = (int64_t)gridDim.x * (blockDim.x >> 5) * 2;
  for (int64_t r = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 2 + half;
       r - half < n_rows; r += step) {
    const bool ok = r < n_rows;
    int64_t g = 0, t = 0;
    if (ok) ra.split(r, g, t);
    uint4 raw = make_uint4(0, 0, 0, 0);
    if (ok) raw = *reinterpret_cast<const uint4*>(v + g * vgs + t * vrs + c * 8);
    const __half* hv = reinterpret_cast<const __half*>(&raw);
    float x[8];
    float lo = INFINITY, hi = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      x[j] = __half2float(hv[j]);
      lo = fminf(lo, x[j]);
      hi = fmaxf(hi, x[j]);
    }
    for (int o = 1; o < lpg; o <<= 1) {
      lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    float sc = __fdiv_rn(__fsub_rn(hi, lo), static_cast<float>(maxq));
    if (sc < 1e-8f) sc = 1e-8f;
    uint32_t bitsw = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float qv = rintf(__fdiv_rn(__fsub_rn(x[j], lo), sc));
      qv = fminf(fmaxf(qv, 0.f), static_cast<float>(maxq));
      bitsw |= static_cast<uint32_t>(qv) << (j * BITS);
    }
    uint32_t* dst = packed + g * pgs + t * prs;
    if (BITS == 4) {
      if (ok) dst[c] = bitsw;
    } else {  // 2-bit: 16 values per word = two lanes
      const uint32_t other = __shfl_xor_sync(0xffffffffu, bitsw, 1);
      if (ok && (c & 1) == 0) dst[c >> 1] = bitsw | (other << 16);
    }
    if (ok && (c % lpg) == 0) {
      scales[g * sgs + t * srs + c / lpg] = sc;
      zeros[g * sgs + t * srs + c / lpg] = lo;
    }
  }
}

// ------------------------------------------------------------- TurboQuant
// rot is staged transposed in shared memory (s_rt[j][i] = R[i][j]) so that
// lane i reads consecutive words when computing r_i = sum_j u_j R[i][j].
__global__ void __launch_bounds__(kWarpsPerCta * 32)
    encode_tq_kernel(const void* v, int vdt, RowAddr ra, int64_t vgs, int64_t vrs, int d,
                     int bits, int mode, int gs, const float* rot, const float* bnd,
                     uint32_t* packed, int64_t pgs, int64_t prs, void* scales, int64_t sgs,
                     int64_t srs) {
  extern __shared__ float s_rt[];  // [d][d]
  __shared__ float s_u[kWarpsPerCta][kMaxD];
  __shared__ float s_r[kWarpsPerCta][kMaxD];
  __shared__ uint8_t s_code[kWarpsPerCta][kMaxD];
  __shared__ float s_b[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nbnd = (1 << bits) - 1;
  for (int e = threadIdx.x; e < d * d; e += blockDim.x) {
    const int i = e / d, j = e - i * d;
    s_rt[j * d + i] = rot[e];
  }
  if (threadIdx.x < nbnd) s_b[threadIdx.x] = bnd[threadIdx.x];
  __syncthreads();
  const int64_t n_rows = ra.n_groups * ra.rpg;
  for (int64_t r = (int64_t)blockIdx.x * kWarpsPerCta + warp; r < n_rows;
       r += (int64_t)gridDim.x * kWarpsPerCta) {
    int64_t g, t;
    ra.split(r, g, t);
    const int64_t vo = g * vgs + t * vrs;
    float ss = 0.f;
    for (int c = lane; c < d; c += 32) {
      const float x = load_as_f32(v, vdt, vo + c);
      s_u[warp][c] = x;
      ss = fmaf(x, x, ss);
    }
    float nrm = 0.f;
    if (mode == 0) {
      nrm = sqrtf(warp_sum(ss));
      const float den = fmaxf(nrm, 1e-8f);
      __syncwarp();
      for (int c = lane; c < d; c += 32) s_u[warp][c] = __fdiv_rn(s_u[warp][c], den);
    }
    __syncwarp();
    for (int i = lane; i < d; i += 32) {
      float acc = 0.f;
      for (int j = 0; j < d; ++j) acc = fmaf(s_u[warp][j], s_rt[j * d + i], acc);
      s_r[warp][i] = acc;
    }
    __syncwarp();
    if (mode == 0) {
      for (int i = lane; i < d; i += 32) {
        const float x = s_r[warp][i];
        int q = 0;
        for (int j = 0; j < nbnd; ++j) q += (x > s_b[j]) ? 1 : 0;
        s_code[warp][i] = static_cast<uint8_t>(q);
      }
      if (lane == 0) reinterpret_cast<float*>(scales)[g * sgs + t * srs] = nrm;
    } else {
      const int ng = d / gs;
      for (int gi = 0; gi < ng; ++gi) {
        float acc = 0.f;
        for (int c = gi * gs + lane; c < (gi + 1) * gs; c += 32)
          acc = fmaf(s_r[warp][c], s_r[warp][c], acc);
        acc = warp_sum(acc);
        const __half s16 = __float2half_rn(sqrtf(acc / static_cast<float>(gs)));
        const float s = __half2float(s16);
        for (int c = gi * gs + lane; c < (gi + 1) * gs; c += 32) {
          const float x = s_r[warp][c];
          int q = 0;
          for (int j = 0; j < nbnd; ++j) q += (x > __fmul_rn(s_b[j], s)) ? 1 : 0;
          s_code[warp][c] = static_cast<uint8_t>(q);
        }
        if (lane == 0) reinterpret_cast<__half*>(scales)[g * sgs + t * srs + gi] = s16;
      }
    }
    __syncwarp();
    pack_row(s_code[warp], d, bits, packed + g * pgs + t * prs, lane);
    __syncwarp();
  }
}

// TurboQuant encode on tensor cores (fp16 values, D = 128, 2 or 4 bits): the
// rotation r = v R^T is an M=16-row x N=128 x K=128 warp MMA chain per 16 rows
// with the rotation split into fp16 hi + lo (fp32 accumulate, about fp32
// accuracy; the reference's own summation order is unspecified BLAS). Rows
// are staged by 16-byte loads; norms / group scales, thresholds and code
// packing run on the accumulator fragments (lane (g, t) holds rows g, g + 8
// and columns 8 n + 2t, 2t + 1 of every 8-column tile n).
constexpr int kTqWarps = 16;
constexpr int kTqStride = 136;  // halves per staged row (128 + 8: conflict-free ldmatrix)

template <int BITS>
__global__ void __launch_bounds__(kTqWarps * 32)
    encode_tq_mma_kernel(const __half* v, RowAddr ra, int64_t vgs, int64_t vrs, int mode, const float* rot, const float* bnd, uint32_t* packed,
                         int64_t pgs, int64_t prs, void* scales, int64_t sgs, int64_t srs) {
  extern __shared__ __align__(16) __half sm_tq[];
  __half* s_rh = sm_tq;                          // [128][kTqStride] rotation, hi
  __half* s_rl = s_rh + 128 * kTqStride;         // [128][kTqStride] rotation, lo
  __half* s_rows = s_rl + 128 * kTqStride;       // [warps][2 buffers][16][kTqStride]
  __shared__ float s_b[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  constexpr int nbnd = (1 << BITS) - 1;
  constexpr int bits = BITS;
  for (int e = threadIdx.x; e < 128 * 128; e += blockDim.x) {
    const int i = e >> 7, j = e & 127;
    const float x = rot[e];
    const __half h = __float2half_rn(x);
    s_rh[i * kTqStride + j] = h;
    s_rl[i * kTqStride + j] = __float2half_rn(x - __half2float(h));
  }
  if (threadIdx.x < nbnd) s_b[threadIdx.x] = bnd[threadIdx.x];
  __syncthreads();
  __half* rows2 = s_rows + warp * 2 * 16 * kTqStride;
  const uint32_t a_off =
      (((lane & 7) + ((lane >> 3) & 1) * 8) * kTqStride + ((lane >> 4) & 1) * 8) * 2;
  const uint32_t bh_base = smem_u32(s_rh) +
                           (((lane & 7) + ((lane >> 4) & 1) * 8) * kTqStride + ((lane >> 3) & 1) * 8) * 2;
  const uint32_t bl_base = bh_base + 128 * kTqStride * 2;
  const int64_t n_rows = ra.n_groups * ra.rpg;
  const int64_t rstep = (int64_t)gridDim.x * kTqWarps * 16;
  // 16 rows into staging buffer `buf` with 16-byte cp.async copies (rows
  // past the end are zero-filled)
  auto stage = [&](int64_t r0, int buf) {
    __half* dst = rows2 + buf * 16 * kTqStride;
    // lanes 0..15 split one row address each; lane l copies 16-byte chunk l % 16
    // of rows l / 16, l / 16 + 2, ...
    int64_t my = -1;
    if (lane < 16 && r0 + lane < n_rows) {
      int64_t gg, tt;
      ra.split(r0 + lane, gg, tt);
      my = gg * vgs + tt * vrs;
    }
    const int cv = lane & 15;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int rr = (lane >> 4) + 2 * m;
      const int64_t base = __shfl_sync(0xffffffffu, my, rr);
      cp_async16(smem_u32(dst + rr * kTqStride + cv * 8), base >= 0 ? v + base + cv * 8 : v,
                 base >= 0 ? 16u : 0u);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  int buf = 0;
  int64_t r0 = ((int64_t)blockIdx.x * kTqWarps + warp) * 16;
  if (r0 < n_rows) stage(r0, 0);
  for (; r0 < n_rows; r0 += rstep, buf ^= 1) {
    // prefetch the next 16 rows while this group is rotated and packed
    if (r0 + rstep < n_rows) {
      stage(r0 + rstep, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncwarp();
    __half* rows = rows2 + buf * 16 * kTqStride;
    const uint32_t a_base = smem_u32(rows) + a_off;
    float nrm_lo = 0.f, nrm_hi = 0.f;  // norms of rows g and g + 8 (mode 0)
    if (mode == 0) {
      // lanes 2r, 2r + 1 sum halves of row r
      const __half* rp = rows + (lane >> 1) * kTqStride + (lane & 1) * 64;
      float ss = 0.f;
      for (int j = 0; j < 64; ++j) {
        const float x = __half2float(rp[j]);
        ss = fmaf(x, x, ss);
      }
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      nrm_lo = sqrtf(__shfl_sync(0xffffffffu, ss, 2 * g));
      nrm_hi = sqrtf(__shfl_sync(0xffffffffu, ss, 2 * (g + 8)));
    }
    float acc[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
#pragma unroll 1
    for (int kk = 0; kk < 8; ++kk) {  // rolled: keeps the kernel in the instruction cache
      uint32_t a0, a1, a2, a3;
      ldsm_x4(a_base + kk * 32, a0, a1, a2, a3);
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        const uint32_t off = (np * 16 * kTqStride + kk * 16) * 2;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(bh_base + off, b0, b1, b2, b3);
        mma_16816(acc[2 * np], a0, a1, a2, a3, b0, b1);
        mma_16816(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
        ldsm_x4(bl_base + off, b0, b1, b2, b3);
        mma_16816(acc[2 * np], a0, a1, a2, a3, b0, b1);
        mma_16816(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // codes; rows g (acc[.][0..1]) and g + 8 (acc[.][2..3])
    uint8_t code[16][4];
    float gsc[2][4];  // group scales of rows g, g + 8 (mode 1)
    if (mode == 0) {
      const float den0 = fmaxf(nrm_lo, 1e-8f), den1 = fmaxf(nrm_hi, 1e-8f);
#pragma unroll
      for (int n = 0; n < 16; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x = __fdiv_rn(acc[n][e], e < 2 ? den0 : den1);
          int q = 0;
#pragma unroll
          for (int j = 0; j < nbnd; ++j) q += (x > s_b[j]) ? 1 : 0;
          code[n][e] = static_cast<uint8_t>(q);
        }
      }
    } else {
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {  // groups of 32 columns = 4 tiles
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int n = 4 * q4; n < 4 * q4 + 4; ++n) {
          s0 = fmaf(acc[n][0], acc[n][0], fmaf(acc[n][1], acc[n][1], s0));
          s1 = fmaf(acc[n][2], acc[n][2], fmaf(acc[n][3], acc[n][3], s1));
        }
        s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
        s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
        const float sc0 = __half2float(__float2half_rn(sqrtf(s0 / 32.f)));
        const float sc1 = __half2float(__float2half_rn(sqrtf(s1 / 32.f)));
        gsc[0][q4] = sc0;
        gsc[1][q4] = sc1;
#pragma unroll
        for (int n = 4 * q4; n < 4 * q4 + 4; ++n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float sc = e < 2 ? sc0 : sc1;
            int q = 0;
#pragma unroll
            for (int j = 0; j < nbnd; ++j) q += (acc[n][e] > __fmul_rn(s_b[j], sc)) ? 1 : 0;
            code[n][e] = static_cast<uint8_t>(q);
          }
        }
      }
    }
    // pack: OR the lanes' fields of each word across t, lane t writes words w % 4 == t
#pragma unroll
    for (int hrow = 0; hrow < 2; ++hrow) {
      const int64_t r = r0 + g + 8 * hrow;
      const bool ok = r < n_rows;
      int64_t gg = 0, tt = 0;
      if (ok) ra.split(r, gg, tt);
      uint32_t* dst = packed + gg * pgs + tt * prs;
      if (bits == 2) {
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          uint32_t word = 0;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int n = 2 * w + h;
            word |= (uint32_t)code[n][2 * hrow] << ((8 * h + 2 * t) * 2);
            word |= (uint32_t)code[n][2 * hrow + 1] << ((8 * h + 2 * t + 1) * 2);
          }
          word |= __shfl_xor_sync(0xffffffffu, word, 1);
          word |= __shfl_xor_sync(0xffffffffu, word, 2);
          if (ok && (w & 3) == t) dst[w] = word;
        }
      } else {
#pragma unroll
        for (int w = 0; w < 16; ++w) {
          uint32_t word = ((uint32_t)code[w][2 * hrow] << (2 * t * 4)) |
                          ((uint32_t)code[w][2 * hrow + 1] << ((2 * t + 1) * 4));
          word |= __shfl_xor_sync(0xffffffffu, word, 1);
          word |= __shfl_xor_sync(0xffffffffu, word, 2);
          if (ok && (w & 3) == t) dst[w] = word;
        }
      }
      if (ok) {
        if (mode == 0) {
          if (t == 0) reinterpret_cast<float*>(scales)[gg * sgs + tt * srs] = hrow ? nrm_hi : nrm_lo;
        } else {
          reinterpret_cast<__half*>(scales)[gg * sgs + tt * srs + t] = __float2half_rn(gsc[hrow][t]);
        }
      }
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------- decode
__global__ void __launch_bounds__(kWarpsPerCta * 32)
    value_decode_kernel(const uint32_t* packed, RowAddr ra, int64_t pgs, int64_t prs, int d,
                        int bits, int gs, const float* levels, const void* scales, int sdt,
                        const float* zeros, int64_t sgs, int64_t srs, const float* rot,
                        void* out, int odt, int64_t ogs, int64_t ors) {
  extern __shared__ float s_rot[];  // [d][d] when rot != nullptr
  __shared__ float s_r[kWarpsPerCta][kMaxD];
  __shared__ float s_lv[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (rot) {
    for (int e = threadIdx.x; e < d * d; e += blockDim.x) s_rot[e] = rot[e];
  }
  if (threadIdx.x < (1 << bits)) s_lv[threadIdx.x] = levels[threadIdx.x];
  __syncthreads();
  const int vpw = vals_per_word(bits);
  const uint32_t m = (1u << bits) - 1u;
  const int64_t n_rows = ra.n_groups * ra.rpg;
  for (int64_t r = (int64_t)blockIdx.x * kWarpsPerCta + warp; r < n_rows;
       r += (int64_t)gridDim.x * kWarpsPerCta) {
    int64_t g, t;
    ra.split(r, g, t);
    const uint32_t* pw = packed + g * pgs + t * prs;
    const int64_t so = g * sgs + t * srs;
    for (int c = lane; c < d; c += 32) {
      const uint32_t code = (pw[c / vpw] >> ((c % vpw) * bits)) & m;
      const int gi = c / gs;
      const float s = sdt == SS_F32 ? reinterpret_cast<const float*>(scales)[so + gi]
                                    : h2f(reinterpret_cast<const uint16_t*>(scales)[so + gi]);
      float x = __fmul_rn(s_lv[code], s);
      if (zeros) x = __fadd_rn(x, zeros[so + gi]);
      s_r[warp][c] = x;
    }
    __syncwarp();
    const int64_t oo = g * ogs + t * ors;
    if (rot) {
      for (int j = lane; j < d; j += 32) {
        float acc = 0.f;
        for (int i = 0; i < d; ++i) acc = fmaf(s_r[warp][i], s_rot[i * d + j], acc);
        store_from_f32(out, odt, oo + j, acc);
      }
    } else {
      for (int c = lane; c < d; c += 32) store_from_f32(out, odt, oo + c, s_r[warp][c]);
    }
    __syncwarp();
  }
}

__global__ void scalar_quantize_kernel(const float* v, int64_t n, const float* bnd, int nb,
                                       uint8_t* out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = v[i];
  int q = 0;
  for (int j = 0; j < nb; ++j) q += (x > bnd[j]) ? 1 : 0;
  out[i] = static_cast<uint8_t>(q);
}

__global__ void pack_kernel(const uint8_t* codes, int64_t n_rows, int d, int bits,
                            uint32_t* packed) {
  const int nw = packed_words(d, bits), vpw = vals_per_word(bits);
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n_rows * nw) return;
  const int64_t r = e / nw;
  const int w = static_cast<int>(e - r * nw);
  const uint32_t m = (1u << bits) - 1u;
  uint32_t word = 0;
  for (int i = 0; i < vpw; ++i) {
    const int c = w * vpw + i;
    if (c < d) word |= (static_cast<uint32_t>(codes[r * d + c]) & m) << (i * bits);
  }
  packed[e] = word;
}

__global__ void unpack_kernel(const uint32_t* packed, int64_t n_rows, int d, int bits,
                              uint8_t* codes) {
  const int nw = packed_words(d, bits), vpw = vals_per_word(bits);
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n_rows * d) return;
  const int64_t r = e / d;
  const int c = static_cast<int>(e - r * d);
  codes[e] = static_cast<uint8_t>((packed[r * nw + c / vpw] >> ((c % vpw) * bits)) &
                                  ((1u << bits) - 1u));
}

int grid_rows(int64_t n_rows) {
  int64_t g = (n_rows + kWarpsPerCta - 1) / kWarpsPerCta;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (g > cap) g = cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace ss

using namespace ss;

extern "C" {

int ss_value_encode_grouped(const void* v, int v_dtype, int64_t n_groups, int64_t rows_per_group,
                            int64_t v_group_stride, int64_t v_row_stride, int d, int bits,
                            int group_size, uint32_t* packed, int64_t p_group_stride,
                            int64_t p_row_stride, float* scales, float* zeros,
                            int64_t s_group_stride, int64_t s_row_stride, void* stream) {
  SS_REQUIRE(v && packed && scales && zeros, "ss_value_encode_grouped: null pointer");
  SS_REQUIRE(bits >= 2 && bits <= 4, "ss_value_encode_grouped: bits must be 2, 3 or 4");
  SS_REQUIRE(d > 0 && d <= kMaxD && group_size > 0 && d % group_size == 0,
             "ss_value_encode_grouped: d must be a multiple of group_size and <= 512");
  SS_REQUIRE(bits == 3 || d % (32 / bits) == 0, "ss_value_encode_grouped: d not packable");
  count_dispatch("ss_value_encode_grouped");
  const int64_t n = n_groups * rows_per_group;
  if (n <= 0) return SS_OK;
  if (v_dtype == SS_F16 && d == 128 && (bits == 2 || bits == 4) && group_size % 8 == 0 &&
      group_size >= 8 &&
      ((reinterpret_cast<uintptr_t>(v) | (uintptr_t)(v_group_stride * 2) |
        (uintptr_t)(v_row_stride * 2)) & 15) == 0) {
    int64_t blocks = (n + 15) / 16;  // 8 warps x 2 rows
    const int64_t cap = 8LL * sm_count();
    if (blocks > cap) blocks = cap;
    auto kern = bits == 2 ? encode_grouped_f16_kernel<2> : encode_grouped_f16_kernel<4>;
    kern<<<static_cast<int>(blocks), 256, 0, as_stream(stream)>>>(
        reinterpret_cast<const __half*>(v), RowAddr{n_groups, rows_per_group}, v_group_stride,
        v_row_stride, group_size, packed, p_group_stride, p_row_stride, scales, zeros,
        s_group_stride, s_row_stride);
    return check_launch("ss_value_encode_grouped");
  }
  encode_grouped_kernel<<<grid_rows(n), kWarpsPerCta * 32, 0, as_stream(stream)>>>(
      v, v_dtype, RowAddr{n_groups, rows_per_group}, v_group_stride, v_row_stride, d, bits,
      group_size, packed, p_group_stride, p_row_stride, scales, zeros, s_group_stride,
      s_row_stride);
  return check_launch("ss_value_encode_grouped");
}

int ss_value_encode_tq(const void* v, int v_dtype, int64_t n_groups, int64_t rows_per_group,
                       int64_t v_group_stride, int64_t v_row_stride, int d, int bits, int mode,
                       int group_size, const float* rot, const float* bnd, uint32_t* packed,
                       int64_t p_group_stride, int64_t p_row_stride, void* scales,
                       int64_t s_group_stride, int64_t s_row_stride, void* stream) {
  SS_REQUIRE(v && rot && bnd && packed && scales, "ss_value_encode_tq: null pointer");
  SS_REQUIRE(bits >= 1 && bits <= 4, "ss_value_encode_tq: bits must be in [1, 4]");
  SS_REQUIRE(mode == 0 || mode == 1, "ss_value_encode_tq: mode must be 0 or 1");
  SS_REQUIRE(d > 0 && d <= 128, "ss_value_encode_tq: d must be <= 128");
  SS_REQUIRE(mode == 0 || (group_size > 0 && d % group_size == 0),
             "ss_value_encode_tq: d must be a multiple of group_size");
  SS_REQUIRE(bits == 3 || bits == 1 || d % (32 / bits) == 0, "ss_value_encode_tq: d not packable");
  SS_REQUIRE(bits != 1, "ss_value_encode_tq: 1-bit packing is not defined by the reference");
  count_dispatch("ss_value_encode_tq");
  const int64_t n = n_groups * rows_per_group;
  if (n <= 0) return SS_OK;
  if (v_dtype == SS_F16 && d == 128 && (bits == 2 || bits == 4) &&
      (mode == 0 || group_size == 32) &&
      ((reinterpret_cast<uintptr_t>(v) | (uintptr_t)(v_group_stride * 2) |
        (uintptr_t)(v_row_stride * 2)) & 15) == 0) {
    const size_t smem_t = (size_t)(2 * 128 + kTqWarps * 2 * 16) * kTqStride * 2;
    auto kern = bits == 2 ? encode_tq_mma_kernel<2> : encode_tq_mma_kernel<4>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_t);
    int64_t blocks = (n + kTqWarps * 16 - 1) / (kTqWarps * 16);
    const int64_t cap = sm_count();
    if (blocks > cap) blocks = cap;
    kern<<<static_cast<int>(blocks), kTqWarps * 32, smem_t, as_stream(stream)>>>(
        reinterpret_cast<const __half*>(v), RowAddr{n_groups, rows_per_group}, v_group_stride,
        v_row_stride, mode, rot, bnd, packed, p_group_stride, p_row_stride, scales,
        s_group_stride, s_row_stride);
    return check_launch("ss_value_encode_tq");
  }
  const size_t smem = (size_t)d * d * 4;
  cudaFuncSetAttribute(encode_tq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  encode_tq_kernel<<<grid_rows(n), kWarpsPerCta * 32, smem, as_stream(stream)>>>(
      v, v_dtype, RowAddr{n_groups, rows_per_group}, v_group_stride, v_row_stride, d, bits,
      mode, group_size, rot, bnd, packed, p_group_stride, p_row_stride, scales, s_group_stride,
      s_row_stride);
  return check_launch("ss_value_encode_tq");
}

int ss_scalar_quantize(const float* v, int64_t n, const float* bnd, int n_bnd, uint8_t* out,
                       void* stream) {
  SS_REQUIRE(v && bnd && out, "ss_scalar_quantize: null pointer");
  SS_REQUIRE(n_bnd >= 0 && n_bnd <= 255, "ss_scalar_quantize: too many boundaries");
  count_dispatch("ss_scalar_quantize");
  if (n <= 0) return SS_OK;
  scalar_quantize_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, as_stream(stream)>>>(
      v, n, bnd, n_bnd, out);
  return check_launch("ss_scalar_quantize");
}

int ss_pack_indices(const uint8_t* codes, int64_t n_rows, int d, int bits, uint32_t* packed,
                    void* stream) {
  SS_REQUIRE(codes && packed, "ss_pack_indices: null pointer");
  SS_REQUIRE(bits >= 2 && bits <= 4, "ss_pack_indices: bits must be 2, 3 or 4");
  SS_REQUIRE(bits == 3 || d % (32 / bits) == 0, "ss_pack_indices: d not divisible");
  count_dispatch("ss_pack_indices");
  const int nw = bits == 3 ? (d + 9) / 10 : d / (32 / bits);
  const int64_t n = n_rows * nw;
  if (n <= 0) return SS_OK;
  pack_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, as_stream(stream)>>>(
      codes, n_rows, d, bits, packed);
  return check_launch("ss_pack_indices");
}

int ss_unpack_indices(const uint32_t* packed, int64_t n_rows, int d, int bits, uint8_t* codes,
                      void* stream) {
  SS_REQUIRE(codes && packed, "ss_unpack_indices: null pointer");
  SS_REQUIRE(bits >= 2 && bits <= 4, "ss_unpack_indices: bits must be 2, 3 or 4");
  count_dispatch("ss_unpack_indices");
  const int64_t n = n_rows * d;
  if (n <= 0) return SS_OK;
  unpack_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, as_stream(stream)>>>(
      packed, n_rows, d, bits, codes);
  return check_launch("ss_unpack_indices");
}

int ss_value_decode(const uint32_t* packed, int64_t n_groups, int64_t rows_per_group,
                    int64_t p_group_stride, int64_t p_row_stride, int d, int bits,
                    int group_size, const float* levels, const void* scales, int scale_dtype,
                    const float* zeros, int64_t s_group_stride, int64_t s_row_stride,
                    const float* rot, void* out, int out_dtype, int64_t out_group_stride,
                    int64_t out_row_stride, void* stream) {
  SS_REQUIRE(packed && levels && scales && out, "ss_value_decode: null pointer");
  SS_REQUIRE(bits >= 2 && bits <= 4, "ss_value_decode: bits must be 2, 3 or 4");
  SS_REQUIRE(d > 0 && d <= kMaxD && group_size > 0 && d % group_size == 0,
             "ss_value_decode: bad d / group_size");
  SS_REQUIRE(!rot || d <= 128, "ss_value_decode: rotation needs d <= 128");
  SS_REQUIRE(scale_dtype == SS_F32 || scale_dtype == SS_F16, "ss_value_decode: bad scale dtype");
  count_dispatch("ss_value_decode");
  const int64_t n = n_groups * rows_per_group;
  if (n <= 0) return SS_OK;
  const size_t smem = rot ? (size_t)d * d * 4 : 0;
  if (smem) {
    cudaFuncSetAttribute(value_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  }
  value_decode_kernel<<<grid_rows(n), kWarpsPerCta * 32, smem, as_stream(stream)>>>(
      packed, RowAddr{n_groups, rows_per_group}, p_group_stride, p_row_stride, d, bits,
      group_size, levels, scales, scale_dtype, zeros, s_group_stride, s_row_stride, rot, out,
      out_dtype, out_group_stride, out_row_stride);
  return check_launch("ss_value_decode");
}

}  // extern "C"
