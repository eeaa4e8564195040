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
