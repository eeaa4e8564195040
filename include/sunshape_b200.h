/*
 * sunshape_b200.h -- C ABI of the B200 (sm_100a) SunShape block-VQ KV-cache
 * hot path. Every entry point takes raw device pointers, explicit sizes and
 * strides (in elements unless named *_bytes) and a cudaStream_t passed as
 * void*. Nothing here allocates device memory, synchronizes the stream or
 * keeps state between calls except where stated (the opt-in dispatch
 * counters and a host-side cache of TMA descriptors).
 *
 * Return value: 0 (SS_OK) on success, otherwise an ss_status code;
 * ss_last_error() gives a human readable message for the calling thread.
 *
 * Reference: gauravsaini/sunshape-mlx (pure Python/MLX; its GPU work is
 * Metal kernel bodies behind Python wrappers). Each function names the
 * reference wrapper (file:line) whose role it takes over. The reference's
 * wrappers return None on failure and the caller falls back to CPU code;
 * these functions instead return an error status, which the Python layer
 * raises as an exception -- there is no fallback.
 */
#ifndef SUNSHAPE_B200_H
#define SUNSHAPE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum ss_status {
  SS_OK = 0,
  SS_ERR_BAD_ARG = 1,      /* null pointer, bad shape/stride/alignment */
  SS_ERR_UNSUPPORTED = 2,  /* valid request the kernels do not implement */
  SS_ERR_CUDA = 3,         /* a CUDA runtime/driver call or launch failed */
  SS_ERR_TIMEOUT = 4,      /* a bounded device-side wait gave up */
  SS_ERR_WORKSPACE = 5     /* workspace pointer null or too small */
};

enum ss_dtype { SS_F32 = 0, SS_F16 = 1, SS_BF16 = 2 };

/* Version of this ABI (major*100 + minor). */
int ss_abi_version(void);
/* Message of the last failing call on this host thread ("" if none). */
const char* ss_last_error(void);
/* Number of SMs of the current device (used to size persistent grids). */
int ss_device_sm_count(void);

/* Dispatch counters (reference: kernels.py:33-47 _KERNEL_STATS). Names are
 * the C entry points; counting is always on and costs one host increment. */
int ss_kernel_stats(char* buf, size_t buf_len); /* "name=count\n" lines */
void ss_reset_kernel_stats(void);

/* --------------------------------------------------------------------------
 * Nearest-centroid assignment (block-VQ quantize).
 * Replaces block_vq_quantize_metal (kernels.py:995-1082) and the NumPy loop
 * of SunShapeBlockCodec.quantize (codec.py:472-514); also the assignment
 * step of k-means (codec.py:84-91).
 *
 * Rows are addressed in two levels so that cache layouts (B, H, T, D) can be
 * read/written in place: row r = g * rows_per_group + t (g < n_groups,
 * t < rows_per_group) reads keys + g*key_group_stride + t*key_row_stride and
 * writes out_idx + g*idx_group_stride + t*idx_row_stride (nb bytes).
 *
 * perm: int32[d] gather applied to each key row before blocking (the
 *       ProfilePerm forward transform, codec.py:273-282) or NULL = identity.
 * centroids: f32 [nb][k][bd], nb = d / bd, k <= 256, bd in {2,4,8,16}.
 * heavy: uint8[nb] mixed-precision mask or NULL. Heavy blocks get index 0
 *        and, if out_heavy != NULL, their permuted values are written as
 *        f16 to out_heavy + g*heavy_group_stride + t*heavy_row_stride, in
 *        heavy-block order (n_heavy * bd halves per row).
 * out_pt: optional f32 passthrough (rows, nb, bd) with row stride nb*bd
 *        (dense, same row order), zero except heavy blocks
 *        (SunShapeQuantized.passthrough_values, codec.py:445-447, 487-490).
 * dist_mode: 0 = sum_d (k_d - c_d)^2 in float32 with NumPy's reduction order
 *        (codec.py:497-499; bit-exact with the reference's CPU quantize);
 *        1 = ||k||^2 + ||c||^2 - 2 k.c as the reference's k-means assignment
 *        evaluates it (codec.py:88-91).
 * Ties resolve to the lowest index (np.argmin / strict '<', kernels.py:1020).
 * -------------------------------------------------------------------------- */
int ss_vq_assign(const void* keys, int key_dtype, int64_t n_groups, int64_t rows_per_group,
                 int64_t key_group_stride, int64_t key_row_stride, int d,
                 const int32_t* perm, const float* centroids, int bd, int k,
                 const uint8_t* heavy, uint8_t* out_idx, int64_t idx_group_stride,
                 int64_t idx_row_stride, uint16_t* out_heavy, int64_t heavy_group_stride,
                 int64_t heavy_row_stride, float* out_pt, int dist_mode, void* stream);

/* ----------------------------------------------------------------------------
 * Cache append (the write half of update_and_fetch, cache.py:156-205): new
 * keys are quantized as ss_vq_assign (dist_mode 0) into the index stream at
 * the write position (heavy blocks into kheavy when given), and the new
 * values are stored as f16 rows. Rows: n_groups groups (batch x kv-head) of
 * `rows` new tokens; destination pointers already point at the write
 * position. Decode-sized appends (<= 4096 rows) are one launch.
 * -------------------------------------------------------------------------- */
typedef struct ss_append_args {
  const void* keys; int key_dtype; int64_t key_group_stride, key_row_stride;
  const void* values; int value_dtype; int64_t value_group_stride, value_row_stride;
  int64_t n_groups, rows;
  int d;
  const int32_t* perm; const float* centroids; int bd, k; const uint8_t* heavy;
  uint8_t* idx; int64_t idx_group_stride, idx_row_stride;
  uint16_t* kheavy; int64_t kheavy_group_stride, kheavy_row_stride;
  uint16_t* v; int64_t v_group_stride, v_row_stride;
} ss_append_args;

int ss_cache_append(const ss_append_args* a, void* stream);

/* Assignment kernel selection (no counterpart in the reference, which has one
 * CPU loop and one Metal kernel): 0 = automatic (tensor-core kernel for
 * >= 16384 rows when bd in {4,8,16}, k in {64,128,192,256}, d <= 128 and key rows are
 * 16-byte aligned; CUDA-core kernel otherwise), 1 = CUDA-core kernel only,
 * 2 = tensor-core kernel or SS_ERR_UNSUPPORTED. Process-wide. Both kernels
 * return the same indices. */
int ss_set_assign_path(int path);

/* Synchronizes the stream, then reads and clears the tensor-core assignment
 * kernel's sticky status: SS_ERR_TIMEOUT if one of its pipeline waits gave
 * up (2 s bound; indices of that launch are then invalid), else SS_OK. */
int ss_vq_assign_check(void* stream);

/* k-means update over one assignment (codec.py:93-101): for every block b and
 * centroid c the float32 sum of the assigned rows, accumulated in row order
 * (np.add.at), divided by the count in float64; empty clusters keep their
 * previous centroid. data: f32 (n, nb*bd) already transformed; assign:
 * uint8 (n, nb). cents_in/cents_out: f32 [nb][k][bd] (may not alias). */
int ss_kmeans_update(const float* data, int64_t n, int nb, int bd, const uint8_t* assign,
                     const float* cents_in, float* cents_out, int k, void* stream);

/* --------------------------------------------------------------------------
 * Gather scores (SunShapeBlockCodec.attention_scores, codec.py:575-637;
 * block_vq_score_metal, kernels.py:59-116):
 *   out[q, t] = sum_b <q_b, C[b, idx[t, b]]>   (float32, no scaling)
 * q: f32 (nq, d) already in codec space; idx: uint8 rows (t stride
 * idx_row_stride bytes). The query x centroid table is built in shared
 * memory. out row stride = out_stride.
 * -------------------------------------------------------------------------- */
int ss_vq_scores(const float* q, int nq, int d, const float* centroids, int bd, int k,
                 const uint8_t* idx, int64_t t, int64_t idx_row_stride, float* out,
                 int64_t out_stride, void* stream);
/* Query x centroid table (SunShapeBlockCodec.precompute_query_centroid_dots,
 * codec.py:553-573): out f32 (nq, nb, k), out[q][b][c] = sum_j q[q][b*bd + j]
 * * centroids[b][c][j], q f32 (nq, d) contiguous, already in codec space. */
int ss_query_centroid_dots(const float* q, int64_t nq, int d, const float* centroids, int bd,
                           int k, float* out, void* stream);
/* Row transform out[r] = x[r] @ m (m f32 (d, d) row-major, fused
 * multiply-adds in i order; x f32 rows of stride x_row_stride; out f32 / f16
 * / bf16 rows of stride out_row_stride; d a power of two <= 128). Replaces
 * the rotation products of rotated-mode codecs (codec.py:273-293) and of
 * the TurboQuant value basis (value_codecs.py:159-177). */
int ss_rotate_rows(const float* x, int64_t rows, int d, int64_t x_row_stride, const float* m,
                   void* out, int out_dtype, int64_t out_row_stride, void* stream);
/* Same gather from a precomputed table qdots f32 (nq, nb, k)
 * (block_vq_score_metal's input, kernels.py:87-116). */
int ss_vq_scores_lut(const float* qdots, int nq, int nb, int k, const uint8_t* idx, int64_t t,
                     int64_t idx_row_stride, float* out, int64_t out_stride, void* stream);

/* Reconstruction (codec.py:516-543): out[t, :] = inv_perm(concat_b C[b,
 * idx[t, b]]), with heavy blocks taken from heavy_vals (f16, heavy-block
 * order) when heavy != NULL. inv_perm NULL = identity. out: f32 or f16
 * (out_dtype), rows addressed like ss_vq_assign. */
int ss_vq_dequant(const uint8_t* idx, int64_t n_groups, int64_t rows_per_group,
                  int64_t idx_group_stride, int64_t idx_row_stride, const float* centroids,
                  int d, int bd, int k, const int32_t* inv_perm, const uint8_t* heavy,
                  const uint16_t* heavy_vals, int64_t heavy_group_stride,
                  int64_t heavy_row_stride, void* out, int out_dtype, int64_t out_group_stride,
                  int64_t out_row_stride, void* stream);

/* --------------------------------------------------------------------------
 * Value encoders (cache append path).
 * Grouped min-max (quantize_values, kernels.py:1173-1228): per group of
 * group_size channels scale = max((max-min)/(2^bits-1), 1e-8), zero = min,
 * q = clip(rint((v - zero)/scale)), packed little-end into uint32 words
 * (pack_indices, kernels.py:1102-1137). bits in {2, 3, 4}.
 * TurboQuant (TurboQuantValueCodec.quantize, value_codecs.py:159-171):
 * mode 0 (reference format): n = ||v||, u = v / max(n, 1e-8), r = u R^T,
 *   idx = #{j : r > bnd_j} with bnd the scaled boundaries, scale_out = n
 *   (f32, one per row);
 * mode 1 (per-group extension): r = v R^T, per group of group_size channels
 *   s = f16(||r_g|| / sqrt(group_size)), idx = #{j : r > bnd_j * s},
 *   scale_out = s (f16 per group).
 * rot: f32 (d, d) row-major R (r = v @ R^T). bnd: f32 boundaries (2^bits-1).
 * Rows addressed like ss_vq_assign; packed/scales/zeros are per row with the
 * given strides (scale/zero strides in elements).
 * -------------------------------------------------------------------------- */
int ss_value_encode_grouped(const void* v, int v_dtype, int64_t n_groups, int64_t rows_per_group,
                            int64_t v_group_stride, int64_t v_row_stride, int d, int bits,
                            int group_size, uint32_t* packed, int64_t p_group_stride,
                            int64_t p_row_stride, float* scales, float* zeros,
                            int64_t s_group_stride, int64_t s_row_stride, void* stream);

int ss_value_encode_tq(const void* v, int v_dtype, int64_t n_groups, int64_t rows_per_group,
                       int64_t v_group_stride, int64_t v_row_stride, int d, int bits, int mode,
                       int group_size, const float* rot, const float* bnd, uint32_t* packed,
                       int64_t p_group_stride, int64_t p_row_stride, void* scales,
                       int64_t s_group_stride, int64_t s_row_stride, void* stream);

/* Scalar boundary quantizer (quantize_scalar_to_indices, kernels.py:453-507):
 * out[i] = #{j : v[i] > bnd[j]} for n contiguous f32 values. */
int ss_scalar_quantize(const float* v, int64_t n, const float* bnd, int n_bnd, uint8_t* out,
                       void* stream);

/* Bit packing (pack_indices / unpack_indices, kernels.py:1102-1163) of
 * n_rows rows of d codes: 2-bit -> d/16 words, 3-bit -> ceil(d/10) words
 * (zero padded), 4-bit -> d/8 words. */
int ss_pack_indices(const uint8_t* codes, int64_t n_rows, int d, int bits, uint32_t* packed,
                    void* stream);
int ss_unpack_indices(const uint32_t* packed, int64_t n_rows, int d, int bits, uint8_t* codes,
                      void* stream);

/* Scalar-quantized value decode (dequantize_values kernels.py:1231-1269 and
 * TurboQuantValueCodec.dequantize value_codecs.py:173-177):
 *   r[c] = level[code_c] * scale[g(c)] + (zeros ? zeros[g(c)] : 0)
 * then, if rot != NULL, out = r @ R. levels: f32 [2^bits]. scale_dtype
 * SS_F32 or SS_F16; groups of group_size channels. out f32 or f16. */
int ss_value_decode(const uint32_t* packed, int64_t n_groups, int64_t rows_per_group,
                    int64_t p_group_stride, int64_t p_row_stride, int d, int bits,
                    int group_size, const float* levels, const void* scales, int scale_dtype,
                    const float* zeros, int64_t s_group_stride, int64_t s_row_stride,
                    const float* rot, void* out, int out_dtype, int64_t out_group_stride,
                    int64_t out_row_stride, void* stream);

/* --------------------------------------------------------------------------
 * Fused decode / multi-query attention over the compressed cache.
 * Replaces the fused kernels fused_attention_metal (kernels.py:142-291),
 * fused_attention_causal_metal (303-446), fused_attention_dequant_metal
 * (588-765), fused_attention_dequant_causal_metal (772-928) and the
 * per-(batch, kv-head, q-head) dispatch loop of sunshape_sdpa
 * (attention.py:166-352), including the hybrid cache's fp16 tail
 * (attention.py:313-328): one launch computes the whole (B, Hq, Tq) output.
 *
 * Semantics (attention.py:199-350): qs = dtype(q * scale) in the query's
 * dtype; scores over compressed tokens are sum_b <P(qs)_b, C[b, idx_b]>
 * (+ exact <qs_b, k_b> over heavy fp16 blocks); over tail tokens
 * <qs, k_tail>; causal: token j visible to query row i iff
 * j <= (Tc + Ttail - Tq) + i; optional additive float mask (Tq, Tc+Ttail);
 * softmax in float32; output = sum p v / sum p (empty -> 0), written in
 * out_dtype. Quantized values are decoded as ss_value_decode; with v_rot
 * the accumulation happens in the rotated basis and is rotated back once.
 *
 * All per-token arrays are addressed by pair = b * hkv + h with a per-pair
 * stride (elements) and must hold at least round_up(tc, 128) rows per pair
 * (cache capacity); the kernel streams whole 128-token tiles.
 * -------------------------------------------------------------------------- */
enum ss_vfmt { SS_V_F16 = 0, SS_V_QUANT = 1, SS_V_VQ = 2 };

typedef struct ss_decode_args {
  /* queries (b, hq, tq, d), element strides */
  const void* q; int q_dtype; int64_t q_sb, q_sh, q_st;
  int b, hq, hkv, tq, d;
  float scale;
  /* codec */
  const int32_t* perm;       /* int32[d] or NULL (identity); applied to qs */
  const float* rot_k;        /* f32 (d,d) rotated-mode transform or NULL */
  const float* centroids;    /* f32 [nb][k][bd] */
  int bd, k;
  const uint8_t* heavy;      /* uint8[nb] or NULL */
  int n_heavy;               /* number of nonzero entries of heavy; 0 scores heavy
                                blocks through their centroids like the reference's
                                cache (which keeps no passthrough values) */
  /* compressed tokens */
  int64_t tc;                /* number of compressed tokens per pair */
  const uint8_t* idx; int64_t idx_pair_stride;         /* bytes; rows nb bytes */
  const uint16_t* kheavy; int64_t kheavy_pair_stride;  /* f16 rows n_heavy*bd */
  int vfmt;                  /* ss_vfmt */
  const uint16_t* v; int64_t v_pair_stride;            /* f16 rows d (SS_V_F16) */
  const uint32_t* vq; int64_t vq_pair_stride;          /* packed rows (SS_V_QUANT) */
  int v_bits, v_group;
  const void* v_scales; int v_scale_dtype; int64_t vs_pair_stride;  /* rows d/v_group */
  const float* v_zeros; int64_t vz_pair_stride;        /* rows d/v_group or NULL */
  float v_levels[16];        /* level table for SS_V_QUANT */
  const float* v_rot;        /* f32 (d,d): value = r @ R, or NULL */
  /* SunShape block-VQ values (SS_V_VQ, value_backend "sunshape", cache.py:785-812):
   * u8 rows of d/v_bd centroid indices; value (codec space) = concat of
   * v_cents[b][idx[b]]; the codec's inverse transform goes in v_rot. d = 128,
   * v_bd in {4, 8, 16}, v_k <= 256. */
  const uint8_t* v_idx; int64_t vi_pair_stride;
  const uint16_t* v_cents;   /* f16 [d/v_bd][v_k][v_bd] */
  int v_bd, v_k;
  /* fp16 tail (hybrid buffer): keys in the original basis; values in the
   * original basis, or already rotated (v R^T) when v_rot is set */
  int64_t ttail;
  const uint16_t* k_tail; const uint16_t* v_tail; int64_t tail_pair_stride;
  /* masking */
  int causal;
  const float* mask; int64_t mask_stride;               /* f32 (tq, tc+ttail) or NULL */
  int mask_mode;             /* 0: additive; 1: keep where mask != 0, else score =
                                -FLT_MAX (boolean masks, attention.py:340-341) */
  /* output (b, hq, tq, d) */
  void* out; int out_dtype; int64_t o_sb, o_sh, o_st;
  /* workspace from ss_decode_workspace_size, zero-filled once before first
   * use; the kernel leaves its counters at zero again on exit. Calls that
   * share a workspace must be stream-ordered. */
  void* workspace; size_t workspace_bytes;
  int max_ctas;              /* 0 = all SMs */
  /* Bound of every device-side wait of this launch in nanoseconds (<= 0:
   * 2 s). A wait that runs out makes the launch give up: the output is then
   * invalid, the workspace's error word and the process error sink (see
   * ss_set_error_sink) report SS_ERR_TIMEOUT. */
  int64_t wait_limit_ns;
  /* Test hook, 0 in normal use: t > 0 makes the producer skip the copies of
   * flattened tile t - 1 while still expecting their bytes, so the waits on
   * that tile run out (exercises the timeout path without a GPU fault). */
  int64_t test_skip_tile;
  /* Optional cache append fused into this call (NULL app_keys: none). The
   * newest app_rows tokens of every (batch, kv-head) pair -- positions
   * tc - app_rows .. tc - 1, already counted in tc -- are not yet in the
   * streams: this call quantizes app_keys into idx (heavy blocks into
   * kheavy) and stores app_values as fp16 rows of v, exactly as
   * ss_cache_append would, before any tile holding them is read (the write
   * half of update_and_fetch, cache.py:156-205, and the attention in one
   * step). Keys/values are (pair, token, d) with the given strides in
   * elements, dtype app_dtype. Supported for fp16 values, no fp16 tail,
   * permutation/identity codecs with 4- or 8-dim blocks and at most 4096
   * appended rows in all; otherwise SS_ERR_UNSUPPORTED (nothing written). */
  const void* app_keys; const void* app_values; int app_dtype;
  int64_t app_key_pair_stride, app_key_row_stride;
  int64_t app_value_pair_stride, app_value_row_stride;
  int64_t app_rows;
} ss_decode_args;

size_t ss_decode_workspace_size(const ss_decode_args* a);
int ss_decode_attn(const ss_decode_args* a, void* stream);
/* ss_decode_attn for callers that cannot allocate device memory (runtimes
 * without an allocator, code confined to another framework's memory pool,
 * hosts that only pass pre-registered input/output buffers). No counterpart
 * in the reference, which never manages device memory itself.
 * Identical results to ss_decode_attn; a->workspace is ignored. The decode
 * scratch is a fixed 8 MiB device array inside this library, held by every
 * GPU that loads it until process exit; problems needing more scratch than
 * ss_decode_workspace_size() allows there are rejected with SS_ERR_WORKSPACE.
 * The first call on a device looks up the array's device address (make it
 * before any stream capture). Every call shares the one array: calls that
 * may overlap on the GPU (different streams, or threads) race. No memory is
 * allocated or freed. */
int ss_decode_attn_noalloc(const ss_decode_args* a, void* stream);

/* Reads and clears the sticky device-side error word of a decode workspace
 * (synchronizes the stream). Returns SS_OK or SS_ERR_TIMEOUT. */
int ss_decode_check(void* workspace, void* stream);

/* ss_decode_check for the fixed scratch array of ss_decode_attn_noalloc on the
 * current device (whose address its callers never see). */
int ss_decode_noalloc_check(void* stream);

/* Process-wide error sink (no counterpart in the reference, whose wrappers
 * return None and fall back): host_word is a page-locked host int (from
 * cudaHostAlloc / cudaMallocHost, visible to the device under unified
 * addressing). Every later launch of the decode and the tensor-core
 * assignment kernels ORs a nonzero code into it when one of its bounded
 * waits gives up (1/2/4/8: decode producer/drain/tile/table waits; 16: the
 * assignment pipeline), with a system-scope atomic, so the host can detect a
 * failed launch by reading the word, without synchronizing. NULL detaches
 * the sink. The caller reads and clears the word. */
int ss_set_error_sink(int* host_word);

/* Bound of the tensor-core assignment kernel's pipeline waits (<= 0: 2 s)
 * and a test hook (skip_tile > 0: the loader never stages tile
 * skip_tile - 1, so the waits on it run out). Process-wide; for tests. */
int ss_set_assign_wait(int64_t wait_limit_ns, int64_t skip_tile);

/* Split-KV partials merge across shards (multi-GPU long context): parts is
 * f32 [n_parts][rows][d + 2] holding (o unnormalized[d], m, l) per row;
 * out[rows][d] = sum_g o_g e^{m_g - m*} / sum_g l_g e^{m_g - m*}, written in
 * out_dtype with row stride out_stride; v_rot optional (d, d) rotation. */
int ss_lse_merge(const float* parts, int n_parts, int64_t rows, int d, const float* v_rot,
                 void* out, int out_dtype, int64_t out_stride, void* stream);

/* Same decode, but returns this shard's unnormalized (o, m, l) rows instead
 * of the output: part_out f32 [b*hq*tq][d + 2]. */
int ss_decode_attn_partial(const ss_decode_args* a, float* part_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SUNSHAPE_B200_H */
