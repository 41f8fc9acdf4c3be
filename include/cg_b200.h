/*
 * card_playing_gym_b200 — C ABI of the B200-native self-play hot path.
 *
 * Plain pointers, sizes and a cudaStream_t passed as void*; no torch types. Every
 * function returns 0 (CG_OK) or an error code and leaves a message for
 * cg_last_error(). Device pointers must live on the current CUDA device; host
 * pointers are rejected by the launch. Nothing here falls back to the CPU.
 *
 * Reference interfaces replaced (paths inside maxrlinder/card_playing_gym):
 *   cardgym/nn/cuda_decode.py:135-151,172-202   decode_attention custom op
 *   cardgym/nn/kv_cache.py:84-105,122-138        KVCache.write_step / copy_rows
 *   cardgym/games/plump/model.py:94-167          PlumpEmbedding.forward (field lookup)
 *   cardgym/nn/trunk.py:285-312,391-429          Trunk.condition / Trunk.forward_ragged
 *   cardgym/nn/model.py:76-89                    SequenceModel.forward_ragged
 *   cardgym/games/plump/model.py:204-217         PlumpActor.policy_logits / player_values
 *   cardgym/rl/ppo.py:75-94                      masked_probabilities / sample_rows
 *   cardgym/rl/selfplay.py:486-567               launch_policies / sample_decisions
 *   cardgym/rl/ppo.py:121-144, rl/trainer.py:634-649   gae_advantages / PPOTrainer._gae
 *   cardgym/rl/ppo.py:28-72, rl/trainer.py:733-802     ppo_terms + _policy_loss (+ autograd)
 *   cardgym/rl/trainer.py:822-850                _value_loss (+ autograd)
 *   cardgym/rl/ppo.py:147-153                    weighted_mean_std
 */
#ifndef CG_B200_H
#define CG_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
enum { CG_F32 = 0, CG_F16 = 1, CG_BF16 = 2 };
/* integer index types (token arrays) */
enum { CG_I16 = 16, CG_I32 = 32, CG_I64 = 64 };
/* trunk arithmetic: fp32 everywhere (CUDA cores), or bf16 GEMM operands with fp32 accumulation (tensor cores) */
enum { CG_PREC_FP32 = 0, CG_PREC_BF16 = 1 };
/* status codes */
enum { CG_OK = 0, CG_ERR_ARGUMENT = 1, CG_ERR_CUDA = 2, CG_ERR_WORKSPACE = 3, CG_ERR_FAULT = 4 };

/* Message of the last failed call on this host thread. */
const char* cg_last_error(void);
/* ABI version (increments on any signature change). */
int cg_version(void);
/* Synchronizes the device, returns and clears the device fault word that kernels set
 * when a bounded wait gives up (0 = no fault). */
int cg_fault_status(int* code_out);
/* Kernel launches this process has issued through the library so far. */
int64_t cg_launch_count(void);
/* Measurement hooks (no reference counterpart): while enabled, every decode-attention
 * launch is bracketed by a pair of CUDA events on its stream (up to `capacity` launches;
 * enabling clears earlier records). cg_attention_timings synchronizes and writes the
 * recorded launch durations in milliseconds; it returns how many it wrote (or -1). */
int cg_attention_profiling(int enable, int capacity);
int cg_attention_timings(float* ms_out, int max_count);
/* The same for the tensor-core dense-layer launches of the bf16 decode step. */
int cg_dense_profiling(int enable, int capacity);
int cg_dense_timings(float* ms_out, int max_count);

/* ---------------------------------------------------------------------------------
 * Decode attention straight from the KV pool.
 * Replaces torch.ops.cardgym.decode_attention (cardgym/nn/cuda_decode.py:135-151):
 *   q [B, H, T, D] contiguous, k/v [R, KVH, L, D] (stride over D == 1), rows [B],
 *   lengths [B] (key length including the row's first new token), span, scale;
 *   query t of row b sees keys < min(lengths[b] + t, span).
 * Beyond the reference: any D that is a multiple of 8 up to 128, any H/KVH group
 * and step count T (fp16/bf16 caches with G <= 16 run on the tensor cores, a row's
 * steps in blocks of floor(16 / G) when G*T > 16), spans up to L, and fp32 / fp16 /
 * bf16 caches. q and out may use their own dtypes; out has q's [B, H, T, D] layout.
 * ------------------------------------------------------------------------------- */
int cg_decode_attention(const void* q, int q_dtype, const void* k_cache, const void* v_cache, int kv_dtype,
                        int64_t kv_stride_row, int64_t kv_stride_head, int64_t kv_stride_pos,
                        const int64_t* rows, const int64_t* lengths, int64_t batch, int heads, int kv_heads,
                        int steps, int head_dim, int span, float scale, void* out, int out_dtype, void* stream);

/* ---------------------------------------------------------------------------------
 * KV pool maintenance (cardgym/nn/kv_cache.py). A layer's pool is [R, KVH, L, D]
 * contiguous; the stacked pool is [n_layers, R, KVH, L, D].
 * ------------------------------------------------------------------------------- */
/* KVCache.write_step (kv_cache.py:84-105): k_new/v_new [B, KVH, T, D] (src_dtype) land on
 * rows[b], positions [B, T] (already clamped by the caller, as the reference does). A row
 * outside [0, capacity) or a position outside [0, max_len) is skipped on the device and sets
 * the fault word (0x110, cg_fault_status), where the reference's indexing would raise. */
int cg_kv_write_step(void* k_layer, void* v_layer, int kv_dtype, int64_t capacity, int kv_heads, int max_len,
                     int head_dim, const int64_t* rows, const int64_t* positions, int64_t batch, int steps,
                     const void* k_new, const void* v_new, int src_dtype, void* stream);

/* KVCache.copy_rows (kv_cache.py:122-138): the first `length` positions of every layer of
 * sources[i] onto targets[i]; overlapping source/target sets are allowed (staged through
 * the workspace, at most cg_kv_copy_rows_workspace_bytes). A pair whose source or target
 * lies outside [0, capacity) is skipped on the device and sets the fault word (0x111). */
int64_t cg_kv_copy_rows_workspace_bytes(int n_layers, int kv_heads, int max_len, int head_dim, int kv_dtype,
                                        int64_t count);
int cg_kv_copy_rows(void* k_pool, void* v_pool, int kv_dtype, int n_layers, int64_t capacity, int kv_heads,
                    int max_len, int head_dim, const int64_t* sources, const int64_t* targets, int64_t count,
                    int length, void* workspace, int64_t workspace_bytes, void* stream);

/* cg_kv_copy_rows for callers that cannot allocate device memory (no counterpart in the
 * reference). A collector loop that overlaps host game stepping with device work cannot
 * call cudaMalloc, which synchronizes the device, and a host that drives this library
 * through the C ABI may have no allocator of its own. This variant stages the rows through
 * a fixed buffer inside the library instead of a caller workspace, and allocates nothing.
 * Limit: the staged bytes, count * n_layers * 2 * kv_heads * length * head_dim * element
 * size, must not exceed cg_kv_copy_rows_noalloc_max_bytes() (16 MiB); larger copies are
 * rejected with CG_ERR_ARGUMENT and should be split into several calls. The buffer is
 * shared by every call in the process on a device: calls whose copies overlap in time on
 * the GPU (on different streams) race with each other. The buffer's device address is
 * looked up per device and CUDA context on every call made outside stream capture (so a
 * cudaDeviceReset or another context is followed); a call inside a capture reuses the
 * address its context recorded, so make the first call on each device, and the first after
 * a reset, before any stream capture. Rows or targets outside [0, capacity) are skipped on
 * the device and set the fault word (0x111, cg_fault_status). */
int64_t cg_kv_copy_rows_noalloc_max_bytes(void);
int cg_kv_copy_rows_noalloc(void* k_pool, void* v_pool, int kv_dtype, int n_layers, int64_t capacity, int kv_heads,
                            int max_len, int head_dim, const int64_t* sources, const int64_t* targets, int64_t count,
                            int length, void* stream);

/* ---------------------------------------------------------------------------------
 * Trunk weights: one device blob. Its fp32 section holds the reference's parameters
 * (cardgym/nn/trunk.py:124-139,259-270 names) at the offsets below; cg_trunk_prepare
 * derives the bf16 tensor-core copies of the GEMM weights into the rest of the blob.
 * ------------------------------------------------------------------------------- */
typedef struct {
  int32_t d_model, n_layers, n_heads, n_kv_heads, d_ff, per_layer_dim;
  int32_t input_norm; /* 1: RMSNorm on the embedding sum (trunk.py:265) */
  int32_t reserved;
  uint64_t value_layers; /* bit l set: block l adds a value embedding to V (trunk.py:58-72) */
} cg_trunk_dims;

enum {
  CG_PART_INPUT_NORM = 0, CG_PART_PLE_CONTEXT, CG_PART_FINAL_W, CG_PART_FINAL_B,
  CG_PART_LN_ATTN_W, CG_PART_LN_ATTN_B, CG_PART_QKV, CG_PART_OUT, CG_PART_LN_MLP_W, CG_PART_LN_MLP_B,
  CG_PART_UP, CG_PART_UP_B, CG_PART_DOWN, CG_PART_DOWN_B, CG_PART_COUNT
};

int64_t cg_trunk_blob_bytes(const cg_trunk_dims* dims);
/* Byte offset of a fp32 tensor in the blob (layer ignored for trunk-wide parts); -1 if absent. */
int64_t cg_trunk_part_offset(const cg_trunk_dims* dims, int part, int layer);
/* Fill the blob's bf16 tensor-core section from its fp32 section. */
int cg_trunk_prepare(const cg_trunk_dims* dims, void* blob, void* stream);

/* ---------------------------------------------------------------------------------
 * Plump field lookup (cardgym/games/plump/model.py:94-167).
 * table: fp32 [field_rows + pattern_rows, width] with the d, PLE and value tables side
 * by side (width = d + ple_width + value_width); rows 0..field_rows-1 are the field
 * rows, then the NA-pattern rows.
 * ------------------------------------------------------------------------------- */
typedef struct {
  int32_t field_count;
  int32_t field_slots[16];
  int32_t field_offsets[16];
  int32_t field_na[16]; /* -1: always present */
  int32_t field_rows, pattern_rows, token_width;
  int32_t slot_type, slot_pattern, slot_hand, hand_slots, trick_win_type;
  int32_t rank_offset, suit_offset, num_cards, num_ranks;
} cg_plump_schema;

/* out [n, width] fp32: the raw lookup sums (x | ple lookup | value lookup). */
int cg_plump_embed(const cg_plump_schema* schema, const float* table, int width, const void* tokens, int token_dtype,
                   int64_t n_tokens, float* out, void* stream);

/* ---------------------------------------------------------------------------------
 * One-hot field bags (cardgym/games/piquet/model.py:255-264 `_onehot_bags`, used by
 * PiquetEmbedding.forward 323-345 and RummyEmbedding): for each of n_tokens tokens, the
 * sum of the table rows its `fields` ids select (id = ids[t * ids_stride + f] + offsets[f];
 * offsets may be NULL for ids that already carry them), each distinct row once, as the
 * reference's `zeros(N, rows).scatter_(1, ids, 1) @ table` with fp32 accumulation.
 * table [rows, width] and out [n_tokens, width] share table_dtype (CG_F32, CG_BF16 or
 * CG_F16: the autocast dtype the reference's GEMM runs in); each sum is rounded once.
 * An id outside [0, rows) sets the device fault word to 0x210 and selects nothing.
 * ------------------------------------------------------------------------------- */
int cg_onehot_bags(const void* ids, int ids_dtype, int64_t n_tokens, int64_t ids_stride, int fields,
                   const int64_t* offsets, const void* table, int table_dtype, int64_t rows, int width, void* out,
                   void* stream);

/* The one-hot field lookup fused into the ragged trunk decode (PiquetEmbedding.forward +
 * SequenceModel.forward_ragged, nn/model.py:76-89; bf16 precision on the tensor-core layers
 * only): the sums of an fp32 table [table_rows, d + ple + value] (plus x_add fp32 [B*T, d] on
 * the x columns when non-NULL: the card-grid summary) go straight into the first dense
 * kernel's inputs, which applies Trunk.condition. ids [B*T rows of ids_stride], as for
 * cg_onehot_bags; the rest as cg_trunk_forward_ragged, with its step workspace. */
int cg_bags_forward_ragged(const cg_trunk_dims* dims, const void* blob, const void* ids, int ids_dtype,
                           int64_t ids_stride, int fields, const int64_t* offsets, const float* table,
                           int64_t table_rows, const float* x_add, int64_t batch, int steps, const int64_t* positions,
                           const int64_t* readout_offsets, const int64_t* rows, int span, void* k_pool, void* v_pool,
                           int kv_dtype, int64_t capacity, int max_len, int precision, void* workspace,
                           int64_t workspace_bytes, float* hidden_out, void* stream);

/* ---------------------------------------------------------------------------------
 * Card grid (cardgym/games/piquet/model.py:180-240 `CardGrid.cards`, with GridBlock
 * 129-177 and GridNorm 118-126; rummy's ledger grid, cardgym/games/rummy/model.py:112-225):
 * a token's 4 * ranks card codes (card = suit * ranks + rank) -> per-card features fp32
 * [n, 4 * ranks, width] after `blocks` residual grid blocks and the final
 * RMSNorm, computed as the reference computes it under bf16 autocast (bf16 GEMM operands,
 * fp32 accumulation, every Linear/matmul output, their sum and the GELU rounded to bf16; the
 * residual grid and the norms in fp32). width 32, hidden 64, blocks <= 4. codes: n rows of
 * codes_stride ids (CG_I16/I32/I64), the card codes first (tokens + CARD_START). A code
 * outside the vocabulary sets the fault word 0x230.
 * The summary projection (a plain [32 * width -> d] Linear) stays with the caller's GEMM.
 * ------------------------------------------------------------------------------- */
typedef struct {
  int32_t width, hidden, kernel, blocks, codes;
  int32_t ranks, circular;   /* 8 ranks, 3 zero-padded taps (piquet) or 13 ranks, 5 circular taps (rummy) */
  const float* code_emb;     /* [codes, width] */
  const float* rank_emb;     /* [ranks, width] */
  const float* norm_w[4];    /* per block: GridNorm gain [width] */
  const float* conv_w[4];    /* along_rank Conv1d weight [hidden, width, 3] */
  const float* conv_b[4];    /* [hidden] */
  const float* across_w[4];  /* across_suits [hidden, width] */
  const float* out_w[4];     /* [width, hidden] */
  const float* out_b[4];     /* [width] */
  const float* final_norm;   /* [width] */
} cg_card_grid_weights;
int cg_card_grid(const cg_card_grid_weights* weights, const void* codes, int codes_dtype, int64_t n,
                 int64_t codes_stride, float* cards, void* stream);

/* ---------------------------------------------------------------------------------
 * Card pointer head (cardgym/games/piquet/model.py:348-363 `CardScorer.forward`, the
 * exchange and play heads of PiquetActor.policy_logits 399-411): one logit per card,
 *   out(GELU(hidden(LayerNorm(query(h)[:, None] + card(grid) + card_id)))).
 * Weights are fp32 device pointers in the reference's [out, in] layout; dim must be 64
 * (score_dim), cards <= 32, card_width <= 32, d_model <= 512.
 * hidden fp32 [n, d_model]; grid [n, cards, card_width] in grid_dtype (CG_F32, CG_BF16,
 * CG_F16); logits fp32 [n, cards]. fp32 arithmetic.
 * ------------------------------------------------------------------------------- */
typedef struct {
  int32_t d_model, card_width, dim, cards;
  const float* query_w;  /* [dim, d_model] */
  const float* query_b;  /* [dim] */
  const float* card_w;   /* [dim, card_width] (no bias) */
  const float* card_id;  /* [cards, dim] */
  const float* norm_w;   /* [dim] LayerNorm, eps 1e-5 */
  const float* norm_b;   /* [dim] */
  const float* hidden_w; /* [dim, dim] */
  const float* hidden_b; /* [dim] */
  const float* out_w;    /* [dim] (the [1, dim] output layer) */
  const float* out_b;    /* [1] */
} cg_card_scorer_weights;
int cg_card_scorer(const cg_card_scorer_weights* weights, const float* hidden, int64_t n, const void* grid, int grid_dtype,
                   float* logits, void* stream);

/* Candidate pointer head (cardgym/games/rummy/model.py:292-357 `CandidateScorer.forward`,
 * RummyActor.policy_logits 391-399): per decision n and candidate c,
 *   candidate = card(Σ grid[cards]) + target(Σ grid[target]) + taken(taken @ grid)
 *             + Σ card_id[cards] + Σ target_id[target] + taken @ taken_id
 *             + kind_emb[kind] + size_emb[#cards != NO_CARD]
 *   logit = out(GELU(hidden(LayerNorm(query(h) + candidate))))
 * kind int64 [n, candidates]; cards/target int64 [n, candidates, list] with NO_CARD = cards
 * as padding; taken fp32 [n, candidates, cards] counts or NULL (the play head); grid
 * [n, cards, card_width]; logits fp32 [n, candidates]. dim 64, card_width <= 32,
 * cards <= 64, list <= 16. Bad ids set the fault word: card 0x220, kind 0x221, size 0x222. */
typedef struct {
  int32_t d_model, card_width, dim, cards, kinds, sizes;
  const float* query_w;   /* [dim, d_model] */
  const float* query_b;   /* [dim] */
  const float* card_w;    /* [dim, card_width] */
  const float* target_w;  /* [dim, card_width] */
  const float* taken_w;   /* [dim, card_width] */
  const float* card_id;   /* [cards, dim] */
  const float* target_id; /* [cards, dim] */
  const float* taken_id;  /* [cards, dim] */
  const float* kind_emb;  /* [kinds, dim] */
  const float* size_emb;  /* [sizes, dim] */
  const float* norm_w;
  const float* norm_b;
  const float* hidden_w;  /* [dim, dim] */
  const float* hidden_b;
  const float* out_w;     /* [dim] */
  const float* out_b;     /* [1] */
} cg_candidate_scorer_weights;
int cg_candidate_scorer(const cg_candidate_scorer_weights* weights, const float* hidden, int64_t n, int candidates,
                        int list, const void* grid, int grid_dtype, const int64_t* kind, const int64_t* cards,
                        const int64_t* target, const float* taken, float* logits, void* stream);

/* ---------------------------------------------------------------------------------
 * Ragged cached decode of the whole trunk (cardgym/nn/trunk.py:391-429, 183-223):
 * appends `steps` tokens to each of `batch` cache rows (rows[b], or b when rows is NULL)
 * at positions[b], and returns the final-normed hidden state of token readout_offsets[b]
 * of each row. k_pool/v_pool are the stacked [n_layers, capacity, KVH, max_len, D] pools.
 * cg_trunk_forward_ragged takes conditioned inputs (Trunk.condition outputs):
 *   x fp32 [B, T, d], ple fp32 [B, T, n_layers, per_layer_dim], values fp32 [B, T, n_value_layers, KVH*D].
 * cg_plump_forward_ragged starts from tokens (SequenceModel.forward_ragged, model.py:76-89).
 * ------------------------------------------------------------------------------- */
int64_t cg_trunk_step_workspace_bytes(const cg_trunk_dims* dims, int64_t batch, int steps, int precision);
int cg_trunk_forward_ragged(const cg_trunk_dims* dims, const void* blob, const float* x, const float* ple,
                            const float* values, int64_t batch, int steps, const int64_t* positions,
                            const int64_t* readout_offsets, const int64_t* rows, int span, void* k_pool,
                            void* v_pool, int kv_dtype, int64_t capacity, int max_len, int precision,
                            void* workspace, int64_t workspace_bytes, float* hidden_out, void* stream);

int64_t cg_plump_step_workspace_bytes(const cg_trunk_dims* dims, int64_t batch, int steps, int precision);
int cg_plump_forward_ragged(const cg_trunk_dims* dims, const void* blob, const cg_plump_schema* schema,
                            const float* table, const void* tokens, int token_dtype, int64_t batch, int steps,
                            const int64_t* positions, const int64_t* readout_offsets, const int64_t* rows, int span,
                            void* k_pool, void* v_pool, int kv_dtype, int64_t capacity, int max_len, int precision,
                            void* workspace, int64_t workspace_bytes, float* hidden_out, void* stream);

/* Trunk.condition alone (trunk.py:285-312): raw lookup [n, d+ple+value] -> x, ple, values. */
int cg_trunk_condition(const cg_trunk_dims* dims, const void* blob, const float* lookup, int64_t n_tokens,
                       float* x_out, float* ple_out, float* values_out, int precision, void* stream);

/* ---------------------------------------------------------------------------------
 * Heads, legal masking and sampling for one wave of decisions
 * (cardgym/games/plump/model.py:204-217; cardgym/rl/selfplay.py:486-567; rl/ppo.py:75-94).
 * heads_blob: fp32; policy head h is W [width[h], d] at weight_offset[h] and b [width[h]]
 * at bias_offset[h]; the value MLP (d -> d GELU -> value_outputs) at value_* offsets.
 * ------------------------------------------------------------------------------- */
typedef struct {
  int32_t d_model, n_policy, value_outputs, max_width;
  int32_t width[8];
  int64_t weight_offset[8], bias_offset[8];
  int64_t value_w1, value_b1, value_w2, value_b2; /* -1 when value_outputs == 0 */
} cg_heads_desc;

/* Per decision i: logits of head head_of[i] on hidden[hidden_rows[i]] (hidden_rows NULL: i),
 * masked softmax over legal[i, :width] (uint8 [D, max_width]), inverse-CDF draw with
 * uniforms[i] (float64) clamped to the last legal action. Outputs (any may be NULL except
 * actions): logits/probs fp32 [D, max_width] (zero past the head's width), actions int64 [D],
 * values fp32 [D, value_outputs]. */
int cg_plump_decide(const cg_heads_desc* desc, const float* heads_blob, const float* hidden,
                    const int64_t* hidden_rows, int64_t decisions, const int32_t* head_of, const uint8_t* legal,
                    const double* uniforms, float* logits_out, float* probs_out, int64_t* actions_out,
                    float* values_out, void* stream);

/* masked_probabilities + sample_rows on given logits [rows, width] fp32 (ppo.py:75-94). */
int cg_masked_sample(const float* logits, const uint8_t* mask, const double* uniforms, int64_t rows, int width,
                     float* probs_out, int64_t* actions_out, void* stream);

/* ---------------------------------------------------------------------------------
 * PPO advantage and loss step.
 * ------------------------------------------------------------------------------- */
/* Undiscounted GAE per game segment, acting-seat column (ppo.py:121-144, trainer.py:634-649):
 * values f64 [N, players] (game g owns rows starts[g]..starts[g+1]-1 in decision order),
 * seats int32 [N], returns f64 [G, players] -> advantages f64 [N]. Bit-exact with the
 * reference's float64 recurrence. */
int cg_gae_segments(const double* values, int players, const int32_t* seats, const int64_t* starts, int64_t games,
                    const double* returns, double gae_lambda, double* advantages_out, void* stream);

/* Sums for the batch-global advantage normalisation (ppo.py:147-153): out[0] = sum w,
 * out[1] = sum w (x - shift), out[2] = sum w (x - shift)^2, in float64, deterministic. */
int64_t cg_weighted_sums_workspace_bytes(int64_t n);
int cg_weighted_sums(const double* values, const double* weights, int64_t n, double shift, double* out3,
                     void* workspace, int64_t workspace_bytes, void* stream);
/* x <- (x - mean) / std in place. */
int cg_normalize(double* values, int64_t n, double mean, double std, void* stream);

/* Device-resident form of the same two passes (no host read between them; the sums may be
 * allreduced on the device in between): the second pass takes its shift, the mean
 * sum w x / sum w, from a first pass's sums shift_sums3 on the device; cg_normalize_from_sums
 * takes mean and std = sqrt(max(second[2] / first[0], 1e-12)) from both passes' sums
 * (mean 0, std 1 without weight), as ppo.py:147-153 computes them. */
int cg_weighted_sums_shifted(const double* values, const double* weights, int64_t n, const double* shift_sums3,
                             double* out3, void* workspace, int64_t workspace_bytes, void* stream);
int cg_normalize_from_sums(double* values, int64_t n, const double* first3, const double* second3, void* stream);

/* The fused per-head PPO objective (ppo.py:28-72 terms; trainer.py:774-797 objective):
 *   L = sum_i w_i * loss_i - alpha * sum_i w_i * eligible_i * normalized_entropy_i
 * logits/old_probs fp32 [rows, width] (row stride `stride`), actions int64, advantages and
 * weights fp32 [rows]. Outputs (each may be NULL): dlogits fp32 [rows, width] = dL/dlogits;
 * row_terms fp32 [rows, 8] = (loss, divergence, entropy, normalized entropy, eligible, ratio,
 * clipped, action log-prob); totals f64 [8] = (sum w loss, sum w, sum w entropy,
 * sum w eligible normalized_entropy, sum w eligible, sum w clipped, sum w divergence, L),
 * reduced deterministically through the workspace. */
int64_t cg_ppo_objective_workspace_bytes(int64_t rows);
int cg_ppo_objective(const float* logits, const float* old_probs, int64_t rows, int width, int64_t stride,
                     const int64_t* actions, const float* advantages, const float* weights, float clip_ratio,
                     float alpha, float* dlogits, float* row_terms, double* totals, void* workspace,
                     int64_t workspace_bytes, void* stream);

/* Dense per-seat zero-sum value regression and its gradient (trainer.py:822-850):
 * prediction/targets fp32 [rows, players_max], players int32 [rows], weights fp32 [rows];
 * grad fp32 [rows, players_max] = dloss/dprediction (may be NULL); totals f64 [4] =
 * (loss, sum w/n sum raw^2, sum w/n sum target^2, sum w). */
int64_t cg_value_loss_workspace_bytes(int64_t rows);
int cg_value_loss(const float* prediction, const float* targets, const int32_t* players, const float* weights,
                  int64_t rows, int players_max, float reward_scale, float* grad, double* totals, void* workspace,
                  int64_t workspace_bytes, void* stream);

/* The PPO baseline's seat values (PPOTrainer._baseline / _recorded_values, trainer.py:556-571,
 * 610-632): decision i reads row flat[i] (or i when flat is NULL) of values fp32 [value_rows,
 * seats]; absolute seat s takes column (s - shift[i]) mod players[i], seats >= players[i] zero.
 * center = 0: values already zero-sum centred (the critic's pending values), prediction = the
 * acting seat's (seat[i]) entry. center = 1: raw recorded values, centred over the active seats
 * in float64 first (the reference's numpy arithmetic), prediction = the centred column 0.
 * state_out f64 [n, seats] and prediction_out f64 [n] (either may be NULL). A row or player
 * count out of range zeroes that decision and sets the fault word (0x400 / 0x401). */
int cg_seat_values(const float* values, int64_t value_rows, int seats, const int64_t* flat, const int64_t* shift,
                   const int64_t* players, const int64_t* seat, int64_t n, int center, double* state_out,
                   double* prediction_out, void* stream);

/* center_zero_sum (cardgym/rl/ppo.py:97-108): fp32 [n, seats] minus the mean over each row's
 * first players[i] seats, padded seats zero. */
int cg_center_zero_sum(const float* values, const int64_t* players, int64_t n, int seats, float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CG_B200_H */
