/*
 * iris_b200.h -- C ABI of the B200 (sm_100a) denoiser kernels for Iris-3B.
 *
 * The reference dispatches its fused kernels from Python through
 * torch.mps.compile_shader (src/iris_metal/kernels.py:309-311) and calls
 * F.linear / F.scaled_dot_product_attention for the rest of the per-step
 * forward (src/iris_metal/model.py:46-52,243-250). This library is what a
 * binding of that path binds instead: plain pointers, sizes and a CUDA stream
 * (cudaStream_t passed as void*). Every entry point
 *   - validates its arguments before launching anything and returns
 *     IRIS_EINVAL (message in iris_last_error()) on a bad call,
 *   - returns IRIS_ECUDA if a CUDA call fails,
 *   - enqueues work on `stream` and never synchronises the host,
 *   - never allocates: the caller owns every input, output and workspace.
 * There is no CPU path: the kernels need an sm_100a device.
 *
 * Element types (the *_dtype arguments): IRIS_F32, IRIS_BF16, IRIS_F16.
 * Row maps (seg_rows, seg_stride, seg_offset): logical row r of an operand is
 * physical row (r / seg_rows) * seg_stride + seg_offset + r % seg_rows, so one
 * stream's rows can live inside a joint [text | image] token buffer. The
 * identity map is (rows, 0, 0).
 */
#ifndef IRIS_B200_H
#define IRIS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IRIS_OK 0
#define IRIS_EINVAL 1
#define IRIS_ECUDA 2

#define IRIS_F32 0
#define IRIS_BF16 1
#define IRIS_F16 2

/* GEMM epilogues */
#define IRIS_EPI_STORE 0  /* out = acc (+ bias)                        */
#define IRIS_EPI_SWIGLU 1 /* out = silu(acc[w1 block]) * acc[w3 block] */
#define IRIS_EPI_GATE 2   /* out = aux * sigmoid(acc)                  */
#define IRIS_EPI_HEADS 3  /* [q | k | v] heads -> normed, rotated head layouts (see iris_heads_epilogue) */
#define IRIS_EPI_ADD 4    /* out += acc (+ bias), f32 out updated in place (residual x + f(x)) */
#define IRIS_EPI_SILU 5   /* out = silu(acc (+ bias))                  */

/* Sequence parallelism over processes (peer memory) */
#define IRIS_MAX_PEERS 8        /* ranks one call may span */
#define IRIS_IPC_HANDLE_BYTES 64 /* bytes of an exported buffer handle */

/* IRIS_EPI_HEADS destinations (iris_heads_epilogue.peer_mode) */
#define IRIS_HEADS_LOCAL 0          /* q_out / k_out / v_out of this process */
#define IRIS_HEADS_PEER_SCATTER 1   /* head h -> rank h / (heads / world): its [b, h % (heads / world), token_offset + t] */
#define IRIS_HEADS_PEER_BROADCAST_KV 2 /* q local as with IRIS_HEADS_LOCAL; k and v -> every rank's [b, h, token_offset + t] */

/* Residual-kernel follow-ups (iris_gated_residual_rms_norm next_mode) */
#define IRIS_NEXT_NONE 0
#define IRIS_NEXT_NORM_MODULATE 1 /* next_out = rms_norm(res) * w * (1 + scale[b]) + shift[b] */
#define IRIS_NEXT_SILU_ADD 2      /* next_out = silu(shift[b] + res)  (timestep re-fuse)   */

/* ---- library ---------------------------------------------------------- */
const char* iris_last_error(void);
int iris_abi_version(void);
/* Reads (and with clear != 0 resets) the device error word of the current
 * device after synchronising `stream`: bit 0 = a kernel's bounded wait timed
 * out, bit 1 = a kernel rejected its arguments on the device. */
int iris_device_error(int clear, unsigned int* value, void* stream);

/* ---- row kernels -------------------------------------------------------- */
/* rms_norm_modulate, src/iris_metal/kernels.py:413-452 (MSL :116-146):
 * out[r] = (rms_norm(x[r]) * weight * (1 + scale[b]) + shift[b]) in out_dtype,
 * b = r / rows_per_batch, modulation rows at b * mod_stride. width % 128 == 0. */
int iris_rms_norm_modulate(const void* x, int x_dtype, int64_t x_seg_rows, int64_t x_seg_stride,
                           int64_t x_seg_offset, void* out, int out_dtype, const float* weight, const float* shift,
                           const float* scale, int64_t mod_stride, int64_t rows, int64_t rows_per_batch,
                           int64_t width, float eps, void* stream);

/* gated_residual_rms_norm_, src/iris_metal/kernels.py:455-480 (MSL :148-175):
 * residual[r] += gate[b] * rms_norm(branch[r]) * weight, in place (fp32);
 * residual and branch rows each go through their row map. With next_mode !=
 * IRIS_NEXT_NONE the updated row also produces the next branch input (see
 * IRIS_NEXT_*), written to next_out through the third row map. */
int iris_gated_residual_rms_norm(float* residual, int64_t res_seg_rows, int64_t res_seg_stride,
                                 int64_t res_seg_offset, const void* branch, int branch_dtype, int64_t br_seg_rows,
                                 int64_t br_seg_stride, int64_t br_seg_offset, const float* weight, const float* gate,
                                 int64_t mod_stride, int64_t rows, int64_t rows_per_batch, int64_t width, float eps,
                                 int next_mode, const float* next_weight, const float* next_shift,
                                 const float* next_scale, int64_t next_mod_stride, void* next_out, int next_out_dtype,
                                 int64_t nx_seg_rows, int64_t nx_seg_stride, int64_t nx_seg_offset, void* stream);

/* The arguments of iris_gated_residual_rms_norm for one stream's rows. */
typedef struct iris_residual_problem {
  float* residual;
  int64_t res_seg_rows, res_seg_stride, res_seg_offset;
  const void* branch;
  int64_t br_seg_rows, br_seg_stride, br_seg_offset;
  const float* weight;
  const float* gate;
  int64_t mod_stride, rows, rows_per_batch;
  int next_mode;
  const float* next_weight;
  const float* next_shift;
  const float* next_scale;
  int64_t next_mod_stride;
  void* next_out;
  int64_t nx_seg_rows, nx_seg_stride, nx_seg_offset;
} iris_residual_problem;

/* 1 or 2 residual updates of one width and dtypes in one launch: the text- and
 * image-stream rows of a dual block (src/iris_metal/model.py:284-289, the
 * reference's gated_residual_rms_norm_ once per stream), each with its own
 * weights, modulation rows and row maps. */
int iris_gated_residual_rms_norm_grouped(const iris_residual_problem* problems, int count, int branch_dtype,
                                         int next_out_dtype, int64_t width, float eps, void* stream);

/* x[r] = rms_norm(x[r]) * weight + add[r % rows_per_batch]  (in place, fp32):
 * TextEmbedder norm + y_pos_embedding, src/iris3b/models/dit.py:263-281. */
int iris_rms_norm_add_rows(float* x, const float* weight, const float* add, int64_t rows, int64_t rows_per_batch,
                           int64_t width, float eps, void* stream);

/* ---- attention inputs --------------------------------------------------- */
/* qk_norm_rope, src/iris_metal/kernels.py:334-397 (MSL :37-84): rows of 128
 * in x[b, n, col_offset + h*128 ...] (row stride row_stride elements) ->
 * per-head RMSNorm * weight, rotary pairs (2i, 2i+1) by cos/sin[offset + n],
 * written to out[b, h, offset + n, :] (out has n_out tokens). */
int iris_qk_norm_rope(const void* x, int x_dtype, int64_t batch, int64_t tokens, int64_t row_stride,
                      int64_t col_offset, int64_t heads, const float* weight, const float* cos, const float* sin,
                      float eps, void* out, int out_dtype, int64_t n_out, int64_t offset, void* stream);

/* One projection [b, n, (heads_q + 2 heads_kv) * 128] (bf16, columns q | k | v,
 * head-major: src/iris3b/models/blocks/single_stream.py:111-117) -> q and k
 * normed + rotated by cos/sin[offset + n], v re-laid, all bf16: q as
 * [b, h, offset + n, 128] of n_out tokens per (b, h), k and v likewise of
 * n_out_kv tokens (the reference does this with qk_norm_rope twice plus a V
 * copy, src/iris_metal/model.py:243-250). head_major = 1 writes
 * [h, b, offset + n, 128] instead: each head's rows of every sample are
 * contiguous, the send layout of a sequence-parallel all-to-all. */
int iris_qkv_heads(const void* qkv, int64_t batch, int64_t tokens, int64_t row_stride, int64_t heads_q,
                   int64_t heads_kv, const float* q_weight, const float* k_weight, const float* cos, const float* sin,
                   float eps, void* q_out, void* k_out, void* v_out, int64_t n_out, int64_t n_out_kv, int64_t offset,
                   int head_major, void* stream);

/* ---- tensor-core kernels ------------------------------------------------ */
/* F.linear in the step (src/iris_metal/model.py:46-52): C = epi(A W^T).
 * A [M, K] (lda), W [N, K] (ldw), bf16, K-major; out [*, ldc] f32 or bf16 via
 * the out row map. SWIGLU: W tiles of 256 rows hold 128 rows of w1 then the
 * matching 128 rows of w3; out has N/2 columns. GATE: aux bf16 [*, ldaux]
 * through the aux row map; out = aux * sigmoid(acc). */
int iris_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw, void* out, int out_dtype, int64_t ldc,
                   int64_t M, int64_t N, int64_t K, int epilogue, const float* bias, const void* aux, int64_t ldaux,
                   int64_t out_seg_rows, int64_t out_seg_stride, int64_t out_seg_offset, int64_t aux_seg_rows,
                   int64_t aux_seg_stride, int64_t aux_seg_offset, void* stream);

/* IRIS_EPI_HEADS: the GEMM's columns are heads_q + 2 heads_kv slots of 128
 * (q | k | v, the layout iris_qkv_heads reads); row m is token position
 * t = out_map(m) % tokens of sample b = out_map(m) / tokens. q and k slots are
 * RMS-normed over their 128 fp32 accumulators times q_weight / k_weight and
 * rotated by cos / sin[t] (pairs (2i, 2i+1)), v is copied; each lands in
 * q_out / k_out / v_out (bf16) at [b, h, t, 128] with n_out (q) or n_out_kv
 * (k, v) positions per (b, h), or at [h, b, t, 128] with head_major = 1.
 * src/iris_metal/model.py:243-250,277-279,304-306 (projection + qk_norm_rope
 * twice + the V copy) in one pass; cos / sin must cover `tokens` rows. */
typedef struct iris_heads_epilogue {
  void* q_out;
  void* k_out;
  void* v_out;
  const float* q_weight;
  const float* k_weight;
  const float* cos;
  const float* sin;
  float eps;
  int head_major;
  int64_t heads_q, heads_kv;
  int64_t tokens, batch;
  int64_t n_out, n_out_kv;
  /* Sequence parallelism (IRIS_HEADS_PEER_*; IRIS_HEADS_LOCAL ignores the rest):
   * the rows are this rank's tokens, written to the ranks' buffers through
   * q_peer / k_peer / v_peer[j] (pointers valid in this process, e.g. from
   * iris_ipc_import) at position token_offset + t of n_dest per (b, h). */
  int peer_mode;
  int world;
  int64_t token_offset, n_dest;
  void* q_peer[IRIS_MAX_PEERS];
  void* k_peer[IRIS_MAX_PEERS];
  void* v_peer[IRIS_MAX_PEERS];
} iris_heads_epilogue;

/* One problem of a grouped launch: the arguments of iris_gemm_bf16 as plain
 * data, plus `heads` for IRIS_EPI_HEADS (null otherwise; `out` is unused then). */
typedef struct iris_gemm_problem {
  const void* a;
  int64_t lda;
  const void* w;
  int64_t ldw;
  void* out;
  int out_dtype;
  int64_t ldc;
  int64_t M, N, K;
  int epilogue;
  const float* bias;
  const void* aux;
  int64_t ldaux;
  int64_t out_seg_rows, out_seg_stride, out_seg_offset;
  int64_t aux_seg_rows, aux_seg_stride, aux_seg_offset;
  const iris_heads_epilogue* heads;
} iris_gemm_problem;

/* 1 to 4 independent GEMMs in one persistent launch (the text- and
 * image-stream linears of a dual block, src/iris_metal/model.py:277-289:
 * same op, separate weights); their output tiles share one tile list. */
int iris_gemm_bf16_grouped(const iris_gemm_problem* problems, int count, void* stream);

/* F.scaled_dot_product_attention, non-causal, unmasked
 * (src/iris_metal/model.py:243-250, src/iris3b/nn/attention.py:61-91):
 * q [b, heads_q, n, 128], k/v [b, heads_kv, n, 128] bf16 contiguous;
 * o[(b * n + i) * o_row_stride + h * 128 + d] bf16. heads_q % heads_kv == 0. */
int iris_flash_attn_fwd(const void* q, const void* k, const void* v, void* o, int64_t batch, int64_t heads_q,
                        int64_t heads_kv, int64_t n, int64_t head_dim, float scale, int64_t o_row_stride,
                        void* stream);

/* The same attention with the block's sigmoid gate applied and each stream's
 * rows written densely (src/iris_metal/model.py:281-283,309): token i < split
 * of sample b goes to row b * split + i of o_text, token i >= split to row
 * b * (n - split) + i - split of o_image; o = attn * sigmoid(gate logit), the
 * bf16 logits read from the same rows of gate_text / gate_image (both null:
 * no gate). split = 0 writes every token to o_image. q holds n queries and
 * k / v hold n_kv keys per (b, h); n_kv may differ from n (a sequence-
 * parallel rank's own queries over the keys of the whole sequence).
 * score_bound: 0, or a bound B >= |q . k| * scale over every query / key pair
 * (QK-normed heads: 128 * max|q gain| * max|k gain| * scale, with a little
 * slack for the bf16 rounding of q and k). Once a query row's running max is
 * within 64 log2 units of B, the row keeps it and skips the row-max pass; a
 * bound below the true scores can overflow that row to inf / NaN. */
int iris_flash_attn_fwd_split(const void* q, const void* k, const void* v, int64_t batch, int64_t heads_q,
                              int64_t heads_kv, int64_t n, int64_t n_kv, int64_t head_dim, float scale,
                              float score_bound, int64_t split, void* o_text, void* o_image, const void* gate_text,
                              const void* gate_image, int64_t row_stride, void* stream);

/* Sequence-parallel attention (no reference counterpart: the reference runs
 * on one device): this rank's heads_q heads over all n = world *
 * tokens_per_rank query positions; each output row goes straight to the rank
 * that owns its token, o_peers[j] (pointers valid in this process), row
 * b * tokens_per_rank + i % tokens_per_rank, columns col0 + h * 128 ... of
 * row_stride bf16. The all-to-all of the attention output, done by the
 * epilogue's stores. score_bound as for iris_flash_attn_fwd_split. */
int iris_flash_attn_fwd_peers(const void* q, const void* k, const void* v, int64_t batch, int64_t heads_q,
                              int64_t heads_kv, int64_t n, int64_t n_kv, int64_t head_dim, float scale,
                              float score_bound, void* const* o_peers, int world, int64_t tokens_per_rank,
                              int64_t col0, int64_t row_stride, void* stream);

/* ---- peer memory (sequence parallelism across processes) ---------------- */
/* No reference counterpart. iris_ipc_export: the IPC handle (IRIS_IPC_HANDLE_BYTES)
 * of the allocation holding device pointer ptr and ptr's offset in it;
 * iris_ipc_import maps another process's handle (base of the allocation; add
 * the offset), iris_ipc_close unmaps it. */
int iris_ipc_export(const void* ptr, void* handle, int64_t* offset);
int iris_ipc_import(const void* handle, void** base);
int iris_ipc_close(void* base);

/* Barrier of the ranks of one sequence-parallel call: writes epoch into slot
 * `rank` of every peer's flags (peer_flags[j], mapped into this process), then
 * waits until every peer j has written at least epoch into flags[j]. Work
 * enqueued on `stream` before the barrier (e.g. epilogue stores into peer
 * buffers) is visible to the peers after theirs returns. A wait longer than
 * timeout_ns gives up and sets bit 0 of the device error word. */
int iris_peer_barrier(unsigned int* flags, void* const* peer_flags, int rank, int world, unsigned int epoch,
                      int64_t timeout_ns, void* stream);

/* ---- pixel stage -------------------------------------------------------- */
/* pixel_rms_norm, src/iris_metal/kernels.py:486-498 (MSL :217-232): bf16 out. */
int iris_pixel_rms_norm(const void* pixels, int pixel_dtype, void* out, const float* weight, int64_t n_pixels,
                        float eps, void* stream);

/* pixel_mlp_, src/iris_metal/kernels.py:527-584 (MSL :235-293): per pixel of
 * 16 channels, pixels += bf16(branch * (1 + scale1) + shift1), RMSNorm,
 * fc1 16->64 + b, exact GELU, fc2 64->16 + b, pixels += bf16(mlp * (1 + scale2)
 * + shift2), next_input = rms_norm(pixels) * next_norm_weight. mods bf16
 * [n, 64] = (scale1, shift1, scale2, shift2); fc weights/biases bf16; pixels
 * bf16 (rounded like the reference) or f32 (kept unrounded). */
int iris_pixel_mlp(void* pixels, int pixel_dtype, const void* branch, const void* mods, const float* norm_weight,
                   const void* fc1_w, const void* fc1_b, const void* fc2_w, const void* fc2_b,
                   const float* next_norm_weight, void* next_input, int64_t n_pixels, float eps, void* stream);

/* The last pixel block fused with FinalLayer (src/iris3b/models/dit.py:53-62)
 * and the fold (dit.py:367-374): same update as iris_pixel_mlp, then
 * v[b, c, y, x] = final_w[c] . rms_norm(pixels) * final_norm_weight + final_b[c]
 * written straight into the [b, 3, H, W] fp32 velocity. The pixels belong to
 * patch tokens [token_start, token_start + tokens) of each sample (all L of
 * them, or one sequence-parallel rank's share); only their pixels of v are
 * written. */
int iris_pixel_mlp_head(void* pixels, int pixel_dtype, const void* branch, const void* mods,
                        const float* norm_weight, const void* fc1_w, const void* fc1_b, const void* fc2_w,
                        const void* fc2_b, const float* final_norm_weight, const float* final_w,
                        const float* final_b, float* v, int64_t batch, int64_t height, int64_t width, int64_t patch,
                        int64_t token_start, int64_t tokens, float eps, void* stream);

/* PixelEmbedder.forward, src/iris3b/nn/embeddings.py:319-328, plus the first
 * block's pixel_rms_norm, for patch tokens l in [token_start, token_start +
 * tokens): pixels[(b, l - token_start), ky * p + kx, :] = W x[b, :, y, x] +
 * bias + pos[y * W + x, :] (pos may be null); normed = bf16
 * rms_norm(pixels) * norm_weight. d_pix == 16; W is [16, channels], 1 to 4
 * input channels (3, or 4 for the depth fine-tune's widened embedder,
 * src/iris3b/downstream/depth.py:30-38). */
int iris_pixel_embed(const float* x, const float* w, const float* bias, const float* pos, void* pixels,
                     int pixel_dtype, void* normed, const float* norm_weight, float eps, int64_t batch,
                     int64_t channels, int64_t height, int64_t width, int64_t patch, int64_t token_start,
                     int64_t tokens, void* stream);

/* ---- layout and conditioning -------------------------------------------- */
/* Patchify, src/iris_metal/model.py:188 / F.unfold in dit.py:326, for patch
 * tokens l = gy * gw + gx in [token_start, token_start + tokens):
 * out[b * tokens + l - token_start, c * p * p + ky * p + kx] = x[b, c, gy * p + ky, gx * p + kx] (bf16 out). */
int iris_patchify(const float* x, void* out, int64_t batch, int64_t channels, int64_t height, int64_t width,
                  int64_t patch, int64_t token_start, int64_t tokens, void* stream);

/* Sequence-parallel (Ulysses) pack / unpack around the all-to-all exchanges
 * (no reference counterpart: the reference runs on one device): for every
 * (i0, i1, i2) < (count0, count1,
 * count2), block_bytes contiguous bytes from src + i0 * src_stride0 + i1 *
 * src_stride1 + i2 * src_stride2 to dst + i0 * dst_stride0 + ... (byte
 * strides; pointers, strides and block_bytes multiples of 16; dst and src
 * must not overlap). */
int iris_block_copy(void* dst, int64_t dst_stride0, int64_t dst_stride1, int64_t dst_stride2, const void* src,
                    int64_t src_stride0, int64_t src_stride1, int64_t src_stride2, int64_t count0, int64_t count1,
                    int64_t count2, int64_t block_bytes, void* stream);

/* Fold of a per-pixel head output, src/iris3b/models/dit.py:367-374:
 * v[b, c, gy * p + ky, gx * p + kx] = out[b * L + gy * gw + gx, ky * p + kx, c] (fp32). */
int iris_unpatchify(const float* out, float* v, int64_t batch, int64_t channels, int64_t height, int64_t width,
                    int64_t patch, void* stream);

/* TimestepEmbedder.timestep_embedding, src/iris3b/nn/embeddings.py:41-45:
 * out[b] = [cos(t_b f_k) | sin(t_b f_k)], f_k = exp(-ln(max_period) k / (freq_dim / 2)). */
int iris_timestep_embedding(const float* t, float* out, int64_t batch, int64_t freq_dim, float max_period,
                            void* stream);

/* Small-M linear for the conditioning MLP and shared adaLN cores
 * (src/iris3b/nn/embeddings.py:47-52, src/iris_metal/model.py:190-192):
 * out[m, n] = act_out(sum_k act_in(x[m, k]) w[n, k] + bias[n]); act 0 = none, 1 = silu. */
int iris_gemv(const float* x, int64_t M, int64_t K, const void* w, int w_dtype, const float* bias, float* out,
              int64_t N, int act_in, int act_out, void* stream);

/* Per-block modulation rows, SharedCoreBias.forward (src/iris3b/nn/modulation.py:284-285):
 * out[j, b, :] = core[b, :] + bias[j, :] for j < n_blocks. */
int iris_add_bias_rows(const float* core, const float* bias, float* out, int64_t batch, int64_t n_blocks,
                       int64_t width, void* stream);

/* ---- text adapter (once per prompt) ------------------------------------- */
/* Attention of the text adapters over short sequences
 * (src/iris3b/nn/embeddings.py:79-142,144-207, SelfAttention
 * src/iris3b/nn/attention.py:94-132 without RoPE): qkv holds seqs * n rows of
 * row_stride bf16, columns [q | k | v] with heads * head_dim each (head h at
 * h * head_dim); for every (sequence s, head h, query i):
 * out[s * n + i, h * head_dim + d] = sum_j softmax_j(scale q_i . k_j) v_j[d]
 * (bf16 out, row stride out_stride). q_gain / k_gain: both null, or per-head
 * RMSNorm gains [head_dim] applied to q and k first (eps). key_mask: null, or
 * uint8 [seqs, n] (1 = real token): key j is attended by query i if
 * key_mask[s, j] != 0 or j == i (pad keys masked, the diagonal kept,
 * embeddings.py:199-205). head_dim % 8 == 0, head_dim <= 128; the sequence's
 * keys and values must fit in shared memory (about n * 4 * head_dim bytes,
 * n <= 436 at head_dim 128). */
int iris_small_attention(const void* qkv, int64_t seqs, int64_t n, int64_t heads, int64_t head_dim,
                         int64_t row_stride, const float* q_gain, const float* k_gain, float eps,
                         const uint8_t* key_mask, float scale, void* out, int64_t out_stride, void* stream);

/* LayerwiseTextEmbedder's layer_pool, src/iris3b/nn/embeddings.py:262-264:
 * out[r, c] = sum_l weight[l] x[r * layers + l, c] + bias[0] (x f32 [rows * layers,
 * width], out bf16 [rows, width]; width % 4 == 0). */
int iris_layer_pool(const float* x, int64_t rows, int64_t layers, int64_t width, const float* weight,
                    const float* bias, void* out, void* stream);

/* ---- tiled restoration (the restoration / 4x upscaling task) -------------- */
/* One tile x tile crop of the [channels, height, width] fp32 image x at (top,
 * left) into out [channels, tile, tile] (the crops that tiled() hands to
 * restore_tile, src/iris3b/downstream/restoration.py:87-101). */
int iris_tile_crop(const float* x, int64_t channels, int64_t height, int64_t width, int64_t top, int64_t left,
                   int64_t tile, float* out, void* stream);

/* The restored tile fused into the image (restore_tile's x - sigma v,
 * src/iris_metal/tasks.py:143-150, weighted by gaussian_window,
 * restoration.py:75-84,96-100): for (i, j) < (tile, tile) and every channel c,
 * out[c, top + i, left + j] += (x[c, top + i, left + j] - sigma v[c, i, j]) * window[i, j];
 * weight[top + i, left + j] += window[i, j] when weight is not null. v may be
 * null (x and out unused): only the weights are accumulated. */
int iris_tile_accumulate(const float* x, int64_t channels, int64_t height, int64_t width, const float* v,
                         int64_t tile, const float* window, int64_t top, int64_t left, float sigma, float* out,
                         float* weight, void* stream);

/* out[c, y, x] /= weight[y, x]: the fused tiles' weighted average (restoration.py:101). */
int iris_tile_normalize(float* out, const float* weight, int64_t channels, int64_t height, int64_t width,
                        void* stream);

/* ---- sampler ------------------------------------------------------------ */
/* One CFG + Euler flow step (src/iris3b/flow/solver.py:72-74 and
 * src/iris3b/sampling.py:129-135): with guided != 0, v holds [uncond; cond]
 * (2 * images rows) and v_g = v_u + cfg_scale (v_c - v_u); clean = x - sigma v_g;
 * if sigma_next < 0 x_out = clean (pre-clamp final sample), else
 * x_out = (1 - sigma_next) clean + sigma_next (x - (1 - sigma) clean) / sigma. */
int iris_cfg_euler(const float* v, const float* x, float* x_out, int64_t images, int64_t per_image, float cfg_scale,
                   float sigma, float sigma_next, int guided, void* stream);

/* One multistep DPM-Solver++ step of FlowDPMSolver (src/iris3b/flow/solver.py:58-109,
 * _model_out + _pred_x0 + _first_order / _second_order): with guided != 0, v holds
 * [uncond; cond] (2 * images rows) and out = v_u + cfg_scale (v_c - v_u), else out = v;
 * x0 = out (predict_x != 0) or x - sigma out; x_out = a x + b x0 + c (x0 - x0_prev),
 * x0 also written to x0_out. First order: a = t / s, b = -(1 - t) expm1(-h), c = 0
 * (x0_prev may be null); second order: a = t / s0, b = -(1 - t) expm1(-h),
 * c = -(1 - t) expm1(-h) / (2 r0). All fp32, [images, per_image] contiguous. */
int iris_dpm_update(const float* v, const float* x, const float* x0_prev, float* x0_out, float* x_out, int64_t images,
                    int64_t per_image, float cfg_scale, int guided, float sigma, int predict_x, float a, float b,
                    float c, void* stream);

/* require_finite, src/iris_metal/model.py:102-110: *flag (device int) = 1 if
 * every x[i] is finite, else 0. */
int iris_all_finite(const float* x, int64_t n, int* flag, void* stream);

/* The raise-rather-than-return-a-bad-result contract of require_finite
 * (src/iris_metal/model.py:102-110) extended to bounded waits, which the
 * reference does not have: if the device error word has a bit of `mask` set
 * (bit 0: a kernel's or a peer barrier's bounded wait gave up, so buffers the
 * result depends on may be stale), x[0..n) is overwritten with NaN. Enqueued
 * after every denoiser call; no host synchronisation. */
int iris_poison_on_error(float* x, int64_t n, unsigned int mask, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* IRIS_B200_H */
