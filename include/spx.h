/*
 * spx.h -- C ABI of the B200 (sm_100a) compressed-KV decode path.
 *
 * This library replaces the compute behind nyssaleo/unsloth-spectral's decode path
 * (paths below are relative to that project):
 *   - spectral decode attention over the three-tier cache
 *       unsloth_spectral/spectral_attention.py:117   spectral_attention_forward
 *       unsloth_spectral/kernels/spectral_attention.py:684  spectral_attention_decode
 *   - the batched randomized SVD + INT8 block compression that feeds the cold tier
 *       unsloth_spectral/rsvd.py:28                   batched_randomized_svd
 *       unsloth_spectral/spectral_cache.py:321        SpectralCache._compress_tensor
 *       unsloth_spectral/spectral_cache.py:481        SpectralCache._quantize_int8_batched
 *   - cold-tier reconstruction and the per-block score/value helpers
 *       unsloth_spectral/spectral_cache.py:557        SpectralCache.get_kv
 *       unsloth_spectral/kernels/spectral_attention.py:456  spectral_score_forward
 *       unsloth_spectral/kernels/spectral_attention.py:604  spectral_value_forward
 *
 * Conventions (all entry points):
 *   - Every pointer in an args struct is a DEVICE pointer unless stated otherwise.
 *   - The caller allocates every output and workspace; the library allocates nothing.
 *   - Work is enqueued on `stream` (a cudaStream_t passed as void*); calls are
 *     asynchronous and re-entrant across streams.  No call synchronises the device.
 *   - Every call returns an spx_status.  Arguments are validated on the host before any
 *     launch; a failing call launches nothing.  No kernel traps or exits.
 *     spx_last_error() returns a thread-local message describing the last failure.
 *
 * Cold-tier layout (one cache = L layers x B sequences x H KV heads, NBc block slots):
 *   codes_k  int8   [L][B][H][NBc][T_blk][RK]   token-major INT8 key coefficients
 *   codes_v  int8   [L][B][H][NBc][T_blk*RV]    INT8 value coefficients, value-tile layout:
 *            code (r, t) of a block at byte ((t/16)*RV + (r ^ ((t/16) & 7)))*16 + pos(t%16),
 *            pos(x) = 4*((x%8)/2) + x%2 + 2*(x/8)  (16-token tiles of [RV][16] bytes,
 *            rows XOR-swizzled, tokens ordered 0,1,8,9,2,3,10,11,...: the layout the tensor
 *            cores read directly)
 *   scale_k  f32    [L][B][H][NBc]              dequantisation scale (coeff = code*scale)
 *   scale_v  f32    [L][B][H][NBc]
 *   basis_k  dtype  [L][B][H][NBc][RK][D]        FP16/BF16/FP32 key basis (Vh rows)
 *   basis_v  dtype  [L][B][H][NBc][RV][D]
 *   block_pos int64 [NBc]                        start position of each block
 *   RK, RV are the stored ranks, padded to multiples of 16 with zero codes/rows.
 * Hot (uncompressed, pre-RoPE) tier:
 *   hot_k, hot_v dtype [L][B][H][HC][D]  with hot_pos int64 [hot_len]
 * Positions are shared by all layers, sequences and heads of one call.
 */
#ifndef SPX_H
#define SPX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SPX_ABI_VERSION 4

#if defined(__GNUC__)
#define SPX_API __attribute__((visibility("default")))
#else
#define SPX_API
#endif

typedef enum spx_status {
  SPX_OK = 0,
  SPX_ERR_NULL = 1,         /* a required pointer is NULL */
  SPX_ERR_SHAPE = 2,        /* inconsistent or out-of-range shape argument */
  SPX_ERR_UNSUPPORTED = 3,  /* valid but unsupported configuration */
  SPX_ERR_ALIGN = 4,        /* pointer not aligned as required (16 bytes) */
  SPX_ERR_WORKSPACE = 5,    /* workspace missing or smaller than required */
  SPX_ERR_EMPTY = 6,        /* decode over an empty cache (no cold block, no hot token) */
  SPX_ERR_CUDA = 7,         /* a CUDA runtime call failed (see spx_last_error) */
  SPX_ERR_DEVICE = 8        /* current device is not sm_100 (B200) */
} spx_status;

typedef enum spx_dtype { SPX_F32 = 0, SPX_F16 = 1, SPX_BF16 = 2 } spx_dtype;

/* Which position indexes the cos/sin tables for cold-tier keys.
 *   DISTANCE: clamp(query_position - key_position, 0)  (spectral_attention.py:198)
 *   ABSOLUTE: key_position                              (kernels/spectral_attention.py:411)
 * The hot tier always uses absolute positions, as both reference paths do. */
typedef enum spx_rope_mode { SPX_ROPE_DISTANCE = 0, SPX_ROPE_ABSOLUTE = 1 } spx_rope_mode;

/* ---------------------------------------------------------------------------------
 * Decode attention.  Replaces spectral_attention.py:117-349 (rope_mode DISTANCE) and
 * kernels/spectral_attention.py:684-857 (rope_mode ABSOLUTE): one query token per
 * (layer, sequence, query head) attends over every cold block then the hot tier, with
 * the reference's keep-mask semantics (mask==0 -> -inf) and float32 softmax.
 * ------------------------------------------------------------------------------- */
typedef struct spx_decode_args {
  int32_t num_layers;      /* L >= 1 independent layers in this call */
  int32_t batch;           /* B */
  int32_t num_q_heads;     /* H_q (multiple of num_kv_heads; q-head h reads KV head h / (H_q/H)) */
  int32_t num_kv_heads;    /* H */
  int32_t head_dim;        /* D: 64 or 128 */
  int32_t block_size;      /* T_blk: 16..1024, multiple of 16 */
  int32_t num_blocks;      /* cold blocks in use (0..block_capacity) */
  int32_t block_capacity;  /* NBc */
  int32_t rank_k;          /* RK: 16, 32, 48 or 64 */
  int32_t rank_v;          /* RV: 16, 32, 48 or 64 */
  int32_t hot_len;         /* hot tokens in use (0..hot_capacity) */
  int32_t hot_capacity;    /* HC */
  int32_t dtype;           /* spx_dtype of q, bases, hot tier and out */
  int32_t rope_mode;       /* spx_rope_mode */
  int32_t rope_tied;       /* 1 when cos[:, :D/2] == cos[:, D/2:] and sin likewise (HF tables) */
  int32_t rope_len;        /* rows of the cos/sin tables */
  int64_t query_position;  /* absolute position of the query token */
  float scale;             /* softmax scale, usually 1/sqrt(D) */
  int32_t mask_stride;     /* row stride (elements) of mask; >= num_blocks*T_blk + hot_len */
  const void* q;           /* dtype [L][B][H_q][D], RoPE already applied at query_position */
  const int8_t* codes_k;
  const int8_t* codes_v;
  const float* scale_k;
  const float* scale_v;
  const void* basis_k;
  const void* basis_v;
  const int64_t* block_pos;
  const void* hot_k;       /* pre-RoPE keys */
  const void* hot_v;
  const int64_t* hot_pos;
  const float* cos_table;  /* f32 [rope_len][D] */
  const float* sin_table;  /* f32 [rope_len][D] */
  const uint8_t* mask;     /* optional keep-mask [B][H_q][mask_stride] over keys in order
                              (cold blocks, then hot); shared by all layers; NULL = none */
  void* out;               /* dtype [L][B][H_q][D] */
  void* workspace;         /* >= spx_decode_workspace_size(args) bytes, 256-byte aligned */
  size_t workspace_bytes;
  const float* rope_freq;  /* optional HOST pointer to head_dim/2 floats: the RoPE frequencies
                              theta_i such that the first-half table entries are
                              cos/sin(position * theta_i) (times one common magnitude, if any).
                              With it (tied tables or DISTANCE mode) the projection kernel can
                              run the cold tier, selected by the environment variable
                              SPX_DECODE_PATH=proj; the reconstruct kernel is the default.  Read
                              during the call only. */
  const int32_t* hot_len_device;  /* optional DEVICE pointer: the hot tier holds
                              min(*hot_len_device, hot_len) tokens, read by the kernels when
                              they run; hot_len is then only the bound that sizes the launch.
                              Lets a caller capture decode steps in a CUDA graph while the
                              hot tier grows.  NULL: hot_len tokens. */
} spx_decode_args;

SPX_API size_t spx_decode_workspace_size(const spx_decode_args* args);
SPX_API int spx_decode_attn(const spx_decode_args* args, void* stream);

/* The cold-tier kernel spx_decode_attn runs for these arguments: SPX_PATH_GENERIC (FP32,
 * any supported shape), SPX_PATH_RECONSTRUCT (keys rebuilt on tensor cores, then rotated
 * per token) or SPX_PATH_PROJECTION (rotation folded into a token-feature table; needs
 * rope_freq); minus the spx_status when the arguments are invalid.  Launches nothing. */
#define SPX_PATH_GENERIC 0
#define SPX_PATH_RECONSTRUCT 1
#define SPX_PATH_PROJECTION 2
SPX_API int spx_decode_path(const spx_decode_args* args);

/* Decode attention for callers that cannot allocate device memory.  This entry point has
 * no counterpart in the reference; it exists for hosts with no device allocator on the
 * decode path -- for example a runtime embedding this library through cgo, JNI or
 * another FFI that owns no CUDA allocator, or a serving loop that may not call
 * cudaMalloc/cudaFree there because those calls can synchronise the device or fail under
 * a fixed memory budget.  It computes exactly what spx_decode_attn computes; the caller
 * still passes every input and the output, but args->workspace and
 * args->workspace_bytes are ignored: the scratch is a fixed array of
 * SPX_NOALLOC_SCRATCH_BYTES built into the library, which every device that loads this
 * part of the library holds until the process exits.  Calls needing more scratch than
 * that (spx_decode_workspace_size) fail with SPX_ERR_WORKSPACE before launching anything.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress,
 * with that device current); make that first call before any stream capture.  All calls
 * on a device share the one array and it keeps the last call's contents, so calls whose
 * GPU work overlaps (other streams, other host threads) race: serialise them.  The
 * address is cached per device ordinal for the life of the process: a cudaDeviceReset,
 * or a non-primary context created with the driver API, is not supported. */
#define SPX_NOALLOC_SCRATCH_BYTES (64u << 20)
SPX_API int spx_decode_attn_noalloc(const spx_decode_args* args, void* stream);

/* ---------------------------------------------------------------------------------
 * Multi-query (prefill) attention over the compressed cache.  Replaces the dense path of
 * integration.py:292-346 (get_kv at spectral_cache.py:557-612, RoPE of the keys at their
 * cached positions with the first half of the tables, softmax(Q K^T * scale + mask) V)
 * without materialising K, V or the scores: key and value tiles are rebuilt from the
 * codes and bases inside the kernel.  Keys are in cache order (cold blocks, then hot).
 * Same cache layout and pointers as spx_decode_args; head_dim 128, f16 or bf16,
 * n_rep in {1,2,4,8}, block_size a multiple of 64, ranks 16..64.
 * ------------------------------------------------------------------------------- */
typedef struct spx_prefill_args {
  int32_t batch, num_q_heads, num_kv_heads, head_dim;
  int32_t q_len;           /* queries per sequence */
  int32_t block_size, num_blocks, block_capacity, rank_k, rank_v, hot_len, hot_capacity;
  int32_t dtype;           /* spx_dtype of q, bases, hot tier and out */
  int32_t rope_len;        /* rows of the cos/sin tables (positions are clamped into range) */
  int32_t causal;          /* 1: a key whose position exceeds the query's position is masked */
  int32_t mask_dtype;      /* SPX_F32 or dtype: element type of mask */
  float scale;             /* softmax scale */
  const void* q;           /* dtype [B][H_q][q_len][D], RoPE already applied */
  const int64_t* q_pos;    /* [q_len] query positions (shared by the batch) */
  const int8_t* codes_k;   /* as spx_decode_args, without the layer dimension */
  const int8_t* codes_v;
  const float* scale_k;
  const float* scale_v;
  const void* basis_k;
  const void* basis_v;
  const int64_t* block_pos;
  const void* hot_k;
  const void* hot_v;
  const int64_t* hot_pos;
  const float* cos_table;  /* f32 [rope_len][D] */
  const float* sin_table;
  const void* mask;        /* optional additive mask: element (b, h, i, j), j over keys in cache
                              order, at b*mask_stride_b + h*mask_stride_h + i*mask_stride_q + j */
  int64_t mask_stride_b, mask_stride_h, mask_stride_q;
  void* out;               /* dtype [B][H_q][q_len][D] */
} spx_prefill_args;

SPX_API int spx_prefill_attn(const spx_prefill_args* args, void* stream);

/* ---------------------------------------------------------------------------------
 * Batched randomized SVD + block compression.  Replaces rsvd.py:28-157 and
 * spectral_cache.py:345-407.  Computes, per matrix M_i [m, n], a rank-k factorisation
 * from the caller's Gaussian sketch omega_i [n, r] (r = k + oversampling) with n_iter
 * power iterations, then optionally C_i = U_i * S_i quantised to INT8 with one scale per
 * matrix (the reference's per-(head, block) scale) and the basis Vh_i in basis_dtype.
 * Power iterations re-orthonormalise each step: same subspace as the reference's
 * un-normalised (M M^T)^q M omega in exact arithmetic, without its float32 loss.
 * ------------------------------------------------------------------------------- */
typedef struct spx_rsvd_args {
  int32_t num_mats;        /* Nb */
  int32_t m;               /* rows: 16..1024 */
  int32_t n;               /* cols: 16..128 */
  int32_t k;               /* target rank: 1..64, k < r */
  int32_t r;               /* sketch width k + oversampling: 2..64, r <= min(m, n) - 2 */
  int32_t n_iter;          /* power iterations: 0..8 */
  int32_t in_dtype;        /* spx_dtype of M */
  const void* M;           /* matrix i at M + i*M_mat_stride elements, rows of n contiguous elements */
  const float* omega;      /* f32 [Nb][n][r] contiguous */
  float* U;                /* optional f32 [Nb][m][k] */
  float* S;                /* optional f32 [Nb][k] */
  float* Vh;               /* optional f32 [Nb][k][n] */
  int64_t M_mat_stride;    /* elements between consecutive matrices (>= m*n; 0 means m*n) */
  int8_t* codes;           /* optional INT8 codes of C = U*S; element (i, t, j) at
                              codes[i*codes_mat_stride + t*codes_t_stride + j*codes_j_stride] */
  int64_t codes_mat_stride;
  int64_t codes_t_stride;
  int64_t codes_j_stride;
  int32_t codes_rank_pad;  /* write zero codes for j in [k, codes_rank_pad) (>= k) */
  int32_t codes_tiled;     /* 1: ignore the t/j strides and write each matrix in the value-tile
                              layout of codes_v (m % 16 == 0, codes_rank_pad % 8 == 0) */
  float* qscale;           /* with codes: scale of matrix i at qscale[i*scale_mat_stride] */
  int64_t scale_mat_stride;
  float* qminmax;          /* optional: (min, max) of C_i at qminmax[i*minmax_mat_stride + {0,1}] */
  int64_t minmax_mat_stride;
  void* basis;             /* optional basis rows (Vh) in basis_dtype at
                              basis[i*basis_mat_stride + j*n + d]; rows k..codes_rank_pad-1 zero */
  int32_t basis_dtype;
  int64_t basis_mat_stride;
  void* workspace;         /* >= spx_rsvd_workspace_size(args) bytes, 256-byte aligned */
  size_t workspace_bytes;
} spx_rsvd_args;

SPX_API size_t spx_rsvd_workspace_size(const spx_rsvd_args* args);
SPX_API int spx_rsvd_compress(const spx_rsvd_args* args, void* stream);

/* ---------------------------------------------------------------------------------
 * Per-group symmetric INT8 quantisation, bit-exact with
 * spectral_cache.py:481-516 (_quantize_int8_batched): scale = max(max|x|, 1e-8)/127,
 * code = round_half_even(x / scale) with IEEE division, minmax = (min x, max x).
 * ------------------------------------------------------------------------------- */
typedef struct spx_quant_args {
  int32_t num_groups;      /* N */
  int64_t group_elems;     /* elements per group */
  const float* x;          /* f32 [N][group_elems] */
  int8_t* codes;           /* [N][group_elems] */
  float* scale;            /* [N] */
  float* minmax;           /* optional [N][2] */
  float* dequant;          /* optional f32 [N][group_elems] = code * scale */
} spx_quant_args;

SPX_API int spx_quantize_int8(const spx_quant_args* args, void* stream);

/* ---------------------------------------------------------------------------------
 * Cold-tier reconstruction X = (code * scale) @ basis, replacing spectral_cache.py:557-612
 * (the bmm per block of get_kv).  Writes tokens [0, num_blocks*T_blk) of
 * out dtype [B][H][out_tokens][D].
 * ------------------------------------------------------------------------------- */
typedef struct spx_reconstruct_args {
  int32_t batch, num_kv_heads, head_dim, block_size, num_blocks, block_capacity;
  int32_t rank;            /* stored (padded) rank */
  int32_t rank_major;      /* 0: codes [..][T_blk][rank] (keys); 1: value-tile layout (values) */
  int32_t dtype;           /* dtype of basis and out */
  int32_t out_tokens;      /* token capacity of out per (b, h) */
  const int8_t* codes;
  const float* scale;
  const void* basis;
  void* out;
} spx_reconstruct_args;

SPX_API int spx_reconstruct(const spx_reconstruct_args* args, void* stream);

/* ---------------------------------------------------------------------------------
 * One block's spectral scores and values from float coefficients, replacing
 * kernels/spectral_attention.py:375-453 (scores, absolute-position RoPE) and :544-601
 * (values).  float32 in, float32 out; all tensors contiguous.
 * ------------------------------------------------------------------------------- */
typedef struct spx_block_score_args {
  int32_t batch, num_q_heads, num_kv_heads, head_dim, block_size, rank, rope_len;
  int64_t start_position;
  const float* q;          /* [B][H_q][D] */
  const float* coeffs;     /* [H][T_blk][rank] */
  const float* basis;      /* [H][rank][D] */
  const float* cos_table;
  const float* sin_table;
  float* scores;           /* [B][H_q][T_blk] */
} spx_block_score_args;

typedef struct spx_block_value_args {
  int32_t batch, num_q_heads, num_kv_heads, head_dim, block_size, rank;
  const float* attn;       /* [B][H_q][T_blk] */
  const float* coeffs;     /* [H][T_blk][rank] */
  const float* basis;      /* [H][rank][D] */
  float* out;              /* [B][H_q][D] */
} spx_block_value_args;

SPX_API int spx_block_scores(const spx_block_score_args* args, void* stream);
SPX_API int spx_block_values(const spx_block_value_args* args, void* stream);

/* ---------------------------------------------------------------------------------
 * RMSNorm of the decode loop's hidden rows, with the residual add fused in front.
 * Replaces the fused RMSNorm that Unsloth's inference loop runs around the patched
 * attention (the reference's rebuilt LlamaModel_fast_forward_inference,
 * unsloth_spectral/integration.py:828-834, walks Unsloth's llama decoder, whose
 * layernorms are Unsloth kernels outside the reference).  Rows of `dim` F16/BF16
 * values, all pointers device pointers, 16-byte aligned, dim a multiple of 8 up to 8192:
 *   h = x (+ residual), rounded to dtype; written to residual_out when residual is given
 *   out = dtype(h * rsqrt(mean(h^2) + eps)) * weight   (product rounded to dtype)
 * residual and residual_out are both NULL or both set; x may alias residual_out.
 * ------------------------------------------------------------------------------- */
SPX_API int spx_rmsnorm(const void* x, const void* residual, const void* weight, void* out, void* residual_out,
                        int64_t rows, int dim, float eps, int dtype, void* stream);

/* ---------------------------------------------------------------------------------
 * Query RoPE of the single-token decode forward: the new token's query rotated at its
 * position (the reference's decode path, unsloth_spectral/integration.py:600-612, rotates
 * it with the tables before spectral_attention_decode), one launch for all sequences and
 * heads.  x: `rows` rows of heads x head_dim values (F32/F16/BF16), consecutive rows
 * x_row_stride elements apart, each row's heads contiguous; cos/sin f32 [rope_len][head_dim]
 * tables, the first half used for both halves (half-split convention); position of row r
 * = pos_device[r * pos_stride] (int64, device; pos_stride 0 broadcasts one position) or
 * pos_host when pos_device is NULL, clamped to the table.  out: [rows][heads][head_dim],
 * contiguous, dtype of x; each product and sum rounded in float32:
 *   out[i] = x[i] c_i - x[i + h] s_i,  out[i + h] = x[i + h] c_i + x[i] s_i,  h = head_dim / 2.
 * ------------------------------------------------------------------------------- */
SPX_API int spx_rope_rows(const void* x, int64_t x_row_stride, const float* cos_table, const float* sin_table,
                          int rope_len, const int64_t* pos_device, int64_t pos_stride, int64_t pos_host, void* out,
                          int rows, int heads, int head_dim, int dtype, void* stream);

/* ---------------------------------------------------------------------------------
 * One decode token appended to the hot tier at its device length: the single-token
 * branch of SpectralCache.append (unsloth_spectral/spectral_cache.py:164-319 appends the
 * new key/value rows to the hot buffers).  k, v: [batch][heads][head_dim] rows (dtype),
 * element (b, h, d) at b * stride_b + h * stride_h + d; hot_k, hot_v: the tier buffers
 * [batch][heads][capacity][head_dim]; hot_pos int64 [capacity]; hot_len: the tier's device
 * int32 length; pos: the token's int64 position (device).  Writes row hot_len and
 * hot_pos[hot_len], then advances hot_len by one, in one launch; a length at or past the
 * capacity writes nothing (the host keeps capacity ahead of the length).
 * ------------------------------------------------------------------------------- */
SPX_API int spx_hot_append(const void* k, const void* v, int64_t k_stride_b, int64_t k_stride_h, int64_t v_stride_b,
                           int64_t v_stride_h, void* hot_k, void* hot_v, int64_t* hot_pos, int32_t* hot_len,
                           const int64_t* pos, int batch, int heads, int head_dim, int capacity, int dtype,
                           void* stream);

/* ---------------------------------------------------------------------------------
 * Utilities.
 * ------------------------------------------------------------------------------- */
SPX_API int spx_abi_version(void);
SPX_API const char* spx_status_string(int status);
SPX_API const char* spx_last_error(void);
/* SPX_OK when the current device is sm_100 (B200); SPX_ERR_DEVICE otherwise. */
SPX_API int spx_check_device(void);

#ifdef __cplusplus
}
#endif
#endif /* SPX_H */
