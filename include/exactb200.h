/* exactb200.h -- C ABI of the B200-native exact integer forward pass.
 *
 * Drop-in boundary for the hot path of novain-shibu/exact-llm: the exact integer model
 * (exact_llm.py IntModel / exact_torch.py TModel / experiments GraphDecoder) and the exact
 * group-128 GEMV operator (experiments/speed_fair_kaggle.py "exact::gemv").  Plain pointers and
 * sizes only; no torch types.  Every entry point returns 0 on success and a non-zero code on
 * failure; exb_last_error() returns the message of the calling thread's last failure.
 *
 * Integer conventions (SPEC.md v0.4 of the reference): activations and logits are int64 Q16;
 * weights int8; group-128 scales int32 (< 2^27); per-channel scales and biases int64.
 * Weight matrices are (N, K) = (out, in) row-major.
 */
#ifndef EXACTB200_H
#define EXACTB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* error codes */
#define EXB_OK 0
#define EXB_EINVAL 1     /* bad argument / size / unsupported shape */
#define EXB_ECUDA 2      /* CUDA runtime error */
#define EXB_EDEVICE 3    /* the device reported a numeric-range, bounds or wait-timeout error */
#define EXB_ENOMEM 4

typedef struct exb_model exb_model;

/* Model architecture.  Mirrors the config dict of exact_llm.open_hf (exact_llm.py:227-230)
 * plus the integer-engine capacities. */
typedef struct exb_config {
  int D, H, KV, hd, I, V, NL;  /* hidden, query heads, KV heads, head dim, MLP, vocab, layers */
  int tie;                     /* 1: the head is the embedding matrix (Qwen2.5-0.5B) */
  int lin_kind;                /* 0: group-128 linears (GQLin), 1: per-channel linears (QLin) */
  int n_experts, topk;         /* MoE (Qwen1.5-MoE): 0 for dense models */
  int moe_I, shared_I;
  int max_batch;               /* sequence slots of the KV cache */
  int max_seq;                 /* KV positions per sequence (Smax) */
  int rope_len;                /* rows of the cos/sin tables (>= max_seq) */
  int emb_shift;               /* x = emb_int8 << emb_shift gives Q16 embeddings */
} exb_config;

const char* exb_last_error(void);
int exb_version(void);

/* --------------------------------------------------------------------- operator level */

/* exact::gemv drop-in (experiments/speed_fair_kaggle.py:686-702):
 * out[n] = sum_g Mg[n,g] * sum_{k in g} x16[k] * wT[n,k]   (int64, exact).
 * Device pointers; K % 128 == 0; 16-byte aligned x16 and wT; launches on `stream`. */
int exb_gemv(const int16_t* x16, const int8_t* wT, const int64_t* Mg, int K, int N, int64_t* out, void* stream);

/* GQLin.__call__ (experiments/speed_fair_kaggle.py:722-725) on R rows of device int64 Q16 input:
 * xq, s = qrow(x); tot = sum_g M_g (xq_g . W_g); y = shr(tot, 28 - s) + b.
 * w_NK int8 (N, K); M_NG int32 (N, K/128); bias int64 (N) or NULL; y int64 (R, N);
 * tot_out int64 (R, N) or NULL.  `scratch` = exb_linear_g128_scratch_bytes(R, K, N) device bytes
 * (quantised rows, shifts, int8 digit planes from 16 rows, and a copy of the scales with rows
 * padded to a multiple of 4 int32 -- the engine's own layout -- when K/128 is not one). */
size_t exb_linear_g128_scratch_bytes(int R, int K, int N);
int exb_linear_g128(const int64_t* x, int R, int K, const int8_t* w_NK, const int32_t* M_NG, const int64_t* bias,
                    int N, int64_t* y, int64_t* tot_out, void* scratch, void* stream);

/* exb_linear_g128 without caller scratch, for callers that cannot allocate device memory: hosts
 * that fix their HBM budget at start-up (every byte reserved for weights and KV caches) and plugin
 * hosts that own the allocator.  No counterpart in the reference (its torch path allocates per
 * call).  Same arguments and bit-identical results as exb_linear_g128, minus `scratch`.
 * The scratch is a fixed array inside the library: every GPU that loads it holds about 24 MiB until
 * exit.  Limits: R * K <= EXB_NOALLOC_MAX_XQ, R <= EXB_NOALLOC_MAX_ROWS and K <= 25600 (else
 * EXB_EINVAL with a message, nothing launched).  From 16 rows with N a multiple of 128 it runs the
 * tcgen05 GEMM (one pass over the weights); below that, or for other N, the CUDA-core GEMV, which
 * reads the weights once per 4 rows.  Alignment: w and x 16 bytes, M 4 bytes (any K/128), y, tot,
 * bias 8 bytes.  The first call on a device looks the array's device address up (make it before
 * any stream capture on that device).  All calls on a device share the array: calls whose GPU work
 * overlaps (different streams, no ordering) race and must be ordered by the caller.  Calls no
 * cudaMalloc, cudaFree or allocating library routine. */
#define EXB_NOALLOC_MAX_XQ (1 << 22)
#define EXB_NOALLOC_MAX_ROWS 4096
int exb_linear_g128_noalloc(const int64_t* x, int R, int K, const int8_t* w_NK, const int32_t* M_NG,
                            const int64_t* bias, int N, int64_t* y, int64_t* tot_out, void* stream);

/* QLin.__call__ (exact_llm.py:89-96) with the per-row drop rule, on device buffers.
 * w_NK int8 (N, K); M int64 (N); acc_out int64 (R, N) is required (the drop rule needs the
 * whole row); scratch of exb_linear_g128_scratch_bytes(R, K, 0) bytes. */
int exb_linear_channel(const int64_t* x, int R, int K, const int8_t* w_NK, const int64_t* M, const int64_t* bias,
                       int N, int64_t* y, int64_t* acc_out, void* scratch, void* stream);

/* --------------------------------------------------------------------- model level */

int exb_model_create(const exb_config* cfg, exb_model** out);
void exb_model_destroy(exb_model* m);

/* Integer tables shipped with the model (SPEC.md section 1): exp (10242 entries, Q24), SiLU and
 * sigmoid (8194 entries, Q16), RoPE cos/sin (rope_len x hd/2, Q16).  Host int64 arrays. */
int exb_model_set_tables(exb_model* m, const int64_t* exp_t, const int64_t* silu_t, const int64_t* sig_t,
                         const int64_t* cos_t, const int64_t* sin_t);

/* Upload one named tensor of the integer artifact from host memory.  Names:
 *   emb (int8 V x D), gf (int64 D), head.w (int8 V x D, untied only), head.M (int64 V),
 *   L{i}.g1 / L{i}.g2 (int64 D),
 *   L{i}.{q,k,v,o,gate,up,down}.w (int8 N x K), .M (int32 N x K/128 group | int64 N channel), .b (int64 N),
 *   MoE: L{i}.{router,sgate,sg,su,sd}.{w,M}, L{i}.e{e}.{g,u,d}.{w,M}. */
int exb_model_set_tensor(exb_model* m, const char* name, const void* host, size_t bytes);

/* Fill every tensor with the seeded synthetic integer generator, directly in HBM. */
int exb_model_generate(exb_model* m, uint64_t seed);

/* Upload done: derive fused layouts and range proofs.  Must precede any forward call. */
int exb_model_finalize(exb_model* m);

/* Empty a sequence slot (its next token gets position 0). */
int exb_seq_reset(exb_model* m, int seq);
int exb_seq_len(exb_model* m, int seq);

/* TModel.forward(ids, cache) (exact_torch.py:171-193) for several sequences at once: row i
 * appends token ids[i] to sequence seqs[i] (rows of one sequence in order).  HOST buffers:
 * logits (n x V int64) may be NULL; next (n int32, greedy argmax, lowest index on ties) may be NULL. */
int exb_forward(exb_model* m, int n, const int32_t* ids, const int32_t* seqs, int64_t* logits, int32_t* next);

/* Greedy generation with the token fed back on the device (GraphDecoder.step loop,
 * experiments/speed_fair_kaggle.py:639-645).  Sequences 0..B-1 continue from their current
 * length with first_ids (B); writes tokens (B x steps, host) and optionally every step's logits
 * (steps x B x V, host) -- NULL skips the copy. */
int exb_generate(exb_model* m, int B, const int32_t* first_ids, int steps, int32_t* tokens, int64_t* logits);

/* Same loop on device buffers only (ids_dev B int32 in, tokens_dev B x steps int32 out), on the
 * model's stream; no host synchronisation. */
int exb_generate_device(exb_model* m, int B, const int32_t* ids_dev, int steps, int32_t* tokens_dev);

/* KV cache export (exact_torch.py:140, 146-149: TModel's cache entries kq, sk, v; the static
 * GraphDecoder cache of experiments/speed_fair_kaggle.py:596-606, 617-618): positions 0..n-1 of
 * sequence slot `seq` at layer `layer`, into HOST buffers (any may be NULL):
 *   k_host  int16 (KV, n, hd)  K after RoPE, per (head, position) row quantised by qrow
 *   ks_host int8  (KV, n)      that row's shift sk
 *   v_host  int32 (KV, n, hd)  V, Q16 (the reference keeps it in int64; |V| < 2^31 is checked)
 * n must not exceed the sequence's length.  Tensor parallel: this rank's KV heads. */
int exb_kv_export(exb_model* m, int layer, int seq, int n, int16_t* k_host, int8_t* ks_host, int32_t* v_host);

/* Trace capture (experiments/prover_commit_cost_gpu_kaggle.py:727-742): when on, every forward
 * row records the raw accumulator of every linear (tot for group-128, acc for per-channel) in
 * call order L0.q,k,v,o,gate,up,down, L1..., head.  exb_trace_row_len gives int64 per row. */
int exb_trace_enable(exb_model* m, int on);
int64_t exb_trace_row_len(exb_model* m);
/* copy the trace of the last forward/decode step's rows (rows x row_len int64) to host */
int exb_trace_read(exb_model* m, int64_t* host, int64_t n);

/* Merkle trace commitment computed on the GPU (experiments/commit_audit_kaggle.py:567-628, which
 * hashes on the host): exb_commit_begin turns trace capture on and logs, for every later forward or
 * decode row of sequence slot `seq` at positions < capacity, its trace row plus the residual
 * stream entering every layer and the final one (X) and every layer's roped K and V rows.
 * exb_commit_root hashes the leaves of positions 0..T-1 in the reference order -- Hb(X[L][t]) for
 * L = 0..NL, then per (L, t) Hb(k acc, v acc), Hb(roped K, V), Hb(q acc), Hb(o, gate, up, down acc),
 * then Hb(head acc) per t, where Hb = SHA-256 over each int64 array's little-endian bytes each
 * followed by "|" -- and builds the Merkle tree (leaf nodes SHA-256("L"+leaf), parents
 * SHA-256("N"+left+right), an odd last node paired with itself); it writes the 32-byte root and,
 * when leaves_host is given, the (5 NL + 2) T leaf digests (leaves_bytes must equal 32 times that).
 * Every position 0..T-1 must have been logged.  Dense single-GPU models. */
int exb_commit_begin(exb_model* m, int seq, int capacity);
int exb_commit_root(exb_model* m, int T, uint8_t* root32, uint8_t* leaves_host, int64_t leaves_bytes);
int exb_commit_end(exb_model* m);

/* Weightless cell verifier on the GPU (experiments/commit_audit_kaggle.py:461-512, 647-705): the
 * verifier's secrets are the Freivalds keys of every linear (exb_freivalds_set_keys, r per linear
 * and prime in trace order -- the reference's make_verifier draws them in that order) and a digest
 * of every embedding row (exb_verifier_emb_keys: r_host = 2 x D values in [0, p)).  It checks
 * cells (layer L, position t) of a committed forward of T positions (root from exb_commit_root or
 * any prover) from opened leaves, without using the weights:
 *   cells    n x 2 int32 (L in 0..NL, t in 0..T-1); ids = the T committed token ids
 *   values   per cell, in the reference's needed() order, the opened int64 arrays:
 *            L < NL: X(L,t)[D] | k acc[KV hd] v acc[KV hd] | for s = 0..t: K(L,s)[KV hd] V(L,s)[KV hd]
 *                    | q acc[H hd] | o acc[D] gate acc[I] up acc[I] down acc[D] | X(L+1,t)[D]
 *            L = NL: X(NL,t)[D] | head acc[V]
 *   proofs   per opened leaf, its Merkle path: depth x 32 bytes, depth = number of halvings of
 *            the (5 NL + 2) T leaves to one root
 *   verdicts 0 accepted; 1000 + j: leaf j of the cell fails its proof; 2 embedding row, 3 k/v,
 *            4 committed K/V row, 5 q, 6 o, 7 gate/up, 8 down, 9 next residual row, 10 head
 *            (the reference's rejection reasons). */
int exb_verifier_emb_keys(exb_model* m, const int32_t* r_host);
int exb_verify_cells(exb_model* m, int T, const uint8_t* root32, int n_cells, const int32_t* cells, const int32_t* ids,
                     const int64_t* values, int64_t n_values, const uint8_t* proofs, int64_t proof_bytes,
                     int32_t* verdicts);

/* Integer sampler on the GPU (exact_llm.py:243-259): y = shr(logit * tnum, 16) with
 * tnum = round(2^16 / temperature); Q20 probabilities p = (e << 20) // sum(e) from the exp table at
 * max(y) - y; token = first index whose running sum of p exceeds (u20 * sum(p)) >> 20, where
 * u20 = splitmix64(seed, position) >> 44.
 *   exb_sample        tokens of R host logits rows (R x V int64), per-row seed and position
 *   exb_sampling      on: the decode steps of exb_generate / exb_generate_device (B <= 4 rows)
 *                     choose row b's next token with seeds[b] at positions[b], which then advance
 *                     by one per step (the reference's generate() samples its t-th token at t);
 *                     off: greedy argmax again.  Single-GPU models.
 *   exb_sampling_positions  read the rows' next sampling positions
 * The receipt chain (SHA-256 over each step's 1.2 MB logits row, exact_llm.py:260-268) is a
 * sequential hash per step and stays on the host (Python shim `generate_sampled`). */
int exb_sample(exb_model* m, const int64_t* logits, int R, int V, const uint64_t* seeds, const int32_t* positions,
               int64_t tnum, int32_t* tokens);
int exb_sampling(exb_model* m, int on, int B, const uint64_t* seeds, const int32_t* positions, int64_t tnum);
int exb_sampling_positions(exb_model* m, int32_t* positions, int B);

/* Freivalds self-check on every linear (experiments/gpu_engine_trace_verify_kaggle.py:803-834):
 * r_host holds, for each linear in trace order, 2 x N values in [0, p) for p = 2^31-1 and
 * 2147483629 (int32).  The device builds d_p = (W*M)^T r_p mod p and, on every later forward,
 * checks sum_n r_n (t_n mod p) == sum_k d_k (xq_k mod p) (mod p) per row and linear. */
int exb_freivalds_set_keys(exb_model* m, const int32_t* r_host, int64_t n);
int exb_freivalds_read_keys(exb_model* m, int32_t* d_host, int64_t n);   /* 2 x K per linear */
int exb_freivalds_enable(exb_model* m, int on);
int exb_freivalds_status(exb_model* m, int64_t* checks, int64_t* failures);

/* Tensor parallelism over NVLink (one process per GPU, NCCL).  The partition follows the
 * reference layer: q/k/v column-split by heads (when the rank count is a multiple of KV, each KV
 * group's query heads split inside a pair of ranks, e.g. 7B TP8 = 4/3 heads), o row-split by the
 * same heads, gate/up column-split and down row-split by 128-groups of I, the head split over the
 * vocabulary.  Per layer four in-graph all-reduces keep the result bit-identical to one GPU:
 * MAX of the attention-output row max (o's qrow), SUM of o's int64 partial sums, MAX of max|h|
 * (down's qrow), SUM of down's partial sums; the greedy token is MAX of the slice maxima, then
 * MIN of the indices holding it.  Integer sums are order-independent, so any NCCL algorithm is
 * exact.  Dense group-128 models; tensors are set and generated in GLOBAL shapes.
 *   exb_tp_plan      this rank's slice: {qh0, qh1, kh0, kh1, ig0, ig1, v0, v1, vmax} (no GPU needed)
 *   exb_tp_unique_id the NCCL unique id rank 0 creates and every rank passes to create_tp
 *   exb_model_create_tp  collective: every rank calls it at the same time */
int exb_tp_plan(const exb_config* cfg, int rank, int size, int32_t* out9);
int exb_tp_unique_id(uint8_t* out128);
int exb_model_create_tp(const exb_config* cfg, int rank, int size, const uint8_t* unique_id, exb_model** out);

/* Engine options (no counterpart in the reference; they change speed, never results):
 *   "tc"      1 (default): forward calls of >= 16 rows run their linears on the tcgen05 tensor-core
 *             GEMM in chunks of 512 rows (256 for MoE); 0: 4-row CUDA-core GEMV passes
 *   "fuse"    decode GEMVs build their own int16 input rows: 1 (default) the qrow of the o and down inputs;
 *             2 also the RMSNorm of the q|k|v, gate|up and head inputs, each CTA computing it whole;
 *             3 the qrow prologues and the RMSNorm finished in the q|k|v, gate|up and head
 *             prologues from the row statistics (max |x|, sum x^2) that the embedding and the o and
 *             down epilogues publish (no norm kernels; dense single-GPU models without commitment
 *             capture or Freivalds, else level 1); 0 separate kernels
 *   "tail"    1: with fuse 1, the RMSNorm + qrow rows of the gate|up input and of the next layer's q|k|v
 *             (or the head's) input are made by the last CTA of the o / down GEMV from the row
 *             statistics (max |x|, sum x^2) their CTAs publish, and layer 0's by the embedding kernel:
 *             no norm kernels in the decode step; 0 (default) separate norm kernels
 *   "attn"    1 (default): decode RoPE + K/V cache write inside the attention kernel; 0 separate
 *   "pattn"   1 (default): prefill chunks of one sequence run the query-tile attention kernel;
 *             0: the per-row kernel
 *   "tcd"     1: decode-step linears on the tcgen05 GEMM (8-row tiles); 0 (default) CUDA-core GEMVs
 *   "tpar"    tensor parallel: 1 (default) the step's all-reduces run as one-shot kernels over the peers'
 *             memory (CUDA IPC mappings over NVLink, bounded flag waits), NCCL where the peers could
 *             not be mapped; 0 NCCL
 *   "tpx"     tensor parallel with "tpar" 1: 1 (default) the decode step's exchanges are fused into the
 *             kernels around them: the attention, gate|up, o and down kernels write their row maxima /
 *             partial sums into every peer's memory and raise a flag; the o / down GEMV prologues and
 *             the norm kernels wait for the peers' flags (bounded) and reduce; 0: all-reduce kernels
 *             (trace, Freivalds and commitment captures always use those)
 *   "tcp"     1 (default): the multi-row tcgen05 GEMM runs on a persistent grid (one CTA per SM walking
 *             the tiles); 0: one CTA per tile.  Process-wide (every model and exb_linear_g128).
 * Cached step graphs are dropped. */
int exb_set_option(exb_model* m, const char* name, int64_t value);

/* MoE models: the router's top-k experts (ties to the lower index) of every row of the last
 * exb_forward call for one layer, as (rows, topk) int32 (rows <= 4096).  Mirrors the reference's
 * per-layer `sel` (experiments/moe_exact_kaggle.py:454-467). */
int exb_moe_selections(exb_model* m, int layer, int32_t* host, int64_t n);

/* kernel launches in the last captured decode-step graph (the count behind bench.py's gpu_launches) */
int exb_step_launches(exb_model* m);

/* device error word: bit 1 |V| >= 2^31 (V cache range), 2 wait timeout, 4 Freivalds, 8 bounds */
int exb_device_errors(exb_model* m, int* bits);

/* Time one layer's fused linear kernel alone: `reps` back-to-back launches on the model's stream
 * between CUDA events; *avg_ms = mean duration of one launch.  which: 0 q|k|v, 1 o, 2 gate|up,
 * 3 down, 4 head.  *bytes = algorithmic bytes one launch must move (weights + scales + activations
 * + outputs). */
int exb_bench_linear(exb_model* m, int layer, int which, int R, int reps, float* avg_ms, double* bytes);

/* Profiling: run one decode step for sequences 0..B-1 kernel by kernel (no graph, no programmatic
 * launch overlap) with a CUDA event after every launch; ms_out[i] = duration of launch i.  The step
 * writes the KV cache at each sequence's current length without advancing it. */
int exb_profile_step(exb_model* m, int B, float* ms_out, int max_n, int* n_out);

/* raw pointers for benchmarks / interop */
void* exb_model_stream(exb_model* m);
size_t exb_model_weight_bytes(exb_model* m);

/* Synthetic tensor generator on the device (same integers as the test oracle's generator).
 * kind: 0 int8 weight, 1 int32 scale, 2 int64 scale, 3 int64 bias, 4 int64 gain. */
int exb_gen_tensor(int kind, uint64_t seed, uint64_t stream_id, int64_t n, int64_t K, void* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif
