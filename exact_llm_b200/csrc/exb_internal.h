// Internal (C++) interfaces between the engine and its kernels.  Not part of the C ABI.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include <string>

namespace exb {

// message returned by exb_last_error() for the calling thread
void set_last_error(const std::string& msg);

// One-time work per device (a kernel's function attributes belong to one device's context): bit d
// is set once device d is done.  Setting an attribute twice is harmless, so the races are benign.
struct DevOnce {
  unsigned long long bits = 0;
  static int dev() { int d = 0; cudaGetDevice(&d); return d & 63; }
  bool done() const { return (__atomic_load_n(&bits, __ATOMIC_ACQUIRE) >> dev()) & 1ull; }
  void set() { __atomic_fetch_or(&bits, 1ull << dev(), __ATOMIC_RELEASE); }
};

enum GenKind { GEN_WEIGHT = 0, GEN_SCALE32 = 1, GEN_SCALE64 = 2, GEN_BIAS = 3, GEN_GAIN = 4 };
cudaError_t gen_tensor(int kind, uint64_t seed, uint64_t stream, int64_t n, int64_t K, void* out, cudaStream_t st);
int64_t isqrt_host(int64_t n);

// One linear layer in HBM.  Weights are (N, K) row-major int8 = one contiguous K-byte row per
// output column.  Group-128 layers carry int32 scales (N, K/128); per-channel layers carry int64
// scales (N,).  For a fused SwiGLU pair the rows are interleaved: row 2j = gate j, 2j+1 = up j.
struct LinW {
  const int8_t* w = nullptr;
  const int32_t* Mg = nullptr;     // group-128 scales (N, ldm), ldm >= K/128, read 4 bytes at a time
  int ldm = 0;                     // row pitch of Mg in int32 (the engine pads it to a multiple of 4)
  const int64_t* Mc = nullptr;     // per-channel scales (N) or nullptr
  const int64_t* b = nullptr;      // bias (N) Q16 or nullptr
  int N = 0, K = 0;
  int mbits = 0;                   // per-channel: bitlen(max M)
  bool nodrop = true;              // per-channel: the drop rule can never trigger (host-proven)
};

// attention
// Fused tensor-parallel exchanges of the decode step (tpx.cuh): the kernel that produces a value
// writes it into every rank's exchange area (peer memory mapped with CUDA IPC) and raises its
// flag there; the kernel that consumes it waits for every peer's flag and reduces locally.
constexpr int TPX_MAX_RANKS = 8;
constexpr int TPX_ROWS = 4;                   // activation rows per decode step (the GEMV pass)
enum TpxType {
  TPX_AMAX_O = 0,    // MAX of the attention output's row max (o's qrow shift)
  TPX_SUM_O = 1,     // SUM of o's partial sums (row-split by heads)
  TPX_AMAX_H = 2,    // MAX of the MLP activation's row max (down's qrow shift)
  TPX_SUM_D = 3,     // SUM of down's partial sums (row-split by groups of I)
};
struct TpX {
  int rank = 0, size = 1;
  int D = 0;                                  // width of the partial-sum rows
  char* base[TPX_MAX_RANKS] = {};             // every rank's exchange area, mapped into this process
  unsigned long long* ep = nullptr;           // (4) this rank's exchange counters, one per type
  int* err = nullptr;                         // device error word (wait timeout)
};
size_t tpx_bytes(int size, int D);

struct AttnArgs {
  const int64_t* qkv = nullptr; int ldqkv = 0;  // (R, (H + 2KV) hd) projected q|k|v (before RoPE)
  const int32_t* row_seq = nullptr;             // (R) sequence slot of each row
  const int32_t* row_pos = nullptr;             // (R) absolute position of each row
  const int32_t* cos_t = nullptr;               // (Tmax, hd/2) Q16
  const int32_t* sin_t = nullptr;
  int16_t* kc = nullptr;                        // K cache (B, KV, Smax, hd) int16 (this layer)
  int8_t* ks = nullptr;                         // K shifts (B, KV, Smax)
  int32_t* vc = nullptr;                        // V cache (B, KV, Smax, hd) int32
  int16_t* qq = nullptr;                        // (R, H, hd) quantised roped q
  int32_t* qs = nullptr;                        // (R, H) q shifts
  const int32_t* exp_t = nullptr;
  int64_t* out = nullptr; int ldo = 0;          // (R, H*hd)
  int R = 0, H = 0, KV = 0, hd = 0, Smax = 0, Tmax = 0;
  int64_t inv = 0;                              // round(2^16 / sqrt(hd))
  unsigned long long* amax_out = nullptr;       // per-row max |out| (atomicMax), for the next qrow
  unsigned int* ticket = nullptr;
  int16_t* xq_out = nullptr; int ldq = 0; int32_t* xs_out = nullptr;   // last CTA: qrow(out) rows
  int64_t* kr_out = nullptr; int64_t ldkr = 0;  // trace commitment: roped K | V rows (R, 2 KV hd)
  int* err = nullptr;
  // tensor parallel: the last CTA publishes the final amax_out rows as exchange TPX_AMAX_O
  // (the exchange description lives in device memory: the argument block stays small)
  const TpX* tpx = nullptr;
  unsigned int* tpx_ticket = nullptr;
};
enum Epi {
  EPI_STORE = 0,     // out[r, n] = requant(tot)
  EPI_RESID = 1,     // out[r, n] += requant(tot)       (residual add)
  EPI_SWIGLU = 2,    // rows interleaved gate/up: out[r, j] = shr(isilu(y_gate) * y_up, 16)
  EPI_RAW = 3,       // raw accumulator only
  EPI_HEAD = 4,      // out[r, n] = requant(acc) (optional) + greedy argmax per row
};

// Work done by the LAST CTA of a GEMV to finish (elected with an atomic ticket, no spinning):
// it turns the kernel's complete output rows into the int16 input rows of the next GEMV.
enum Tail {
  TAIL_NONE = 0,
  TAIL_NORM = 1,     // xq, s = qrow(irms(tail_x, tail_gain))      (after a residual add)
  TAIL_QUANT = 2,    // xq = clip(shr(tail_x, s)), s from tail_amax (published by this kernel)
  TAIL_ROPE = 3,     // RoPE + KV-cache write + query rows (after the q|k|v GEMV)
};

// How a GEMV obtains its int16 activation rows (every CTA stages all R rows in shared memory).
enum XIn {
  XIN_Q16 = 0,       // xq (R, ldx) int16 + shifts xs (R), already quantised
  XIN_NORM = 1,      // x64 rows: xq, s = qrow(irms(x, gain))          (every CTA computes it)
  XIN_QUANT = 2,     // x64 rows: xq = clip(shr(x, s)), s from the producer's published max |x|
  XIN_NORMST = 3,    // x64 rows: xq, s = qrow(irms(x, gain)) from the producers' published row
                     // statistics (max |x|, sum x^2): one reduction per CTA instead of three
};

struct GemvArgs {
  const int16_t* xq = nullptr;     // XIN_Q16: (R, ldx) int16 activations
  const int32_t* xs = nullptr;     // XIN_Q16: (R) qrow shifts
  int ldx = 0;
  int xin = XIN_Q16;
  const int64_t* x64 = nullptr; int ldx64 = 0;  // XIN_NORM / XIN_QUANT source rows (int64 Q16)
  const int64_t* gain = nullptr;                // XIN_NORM gains
  const unsigned long long* amax_in = nullptr;  // XIN_QUANT per-row max |x|
  const unsigned long long* nstat_in = nullptr; // XIN_NORMST per-row (max |x|, sum x^2), 2 words per row
  int rb = 0;                                   // columns per warp block (0: chosen by the launcher)
  int pre = -1;                                 // first load batch copied to shared memory before the
                                                // PDL wait: -1 where two CTAs per SM still fit, 0 never
  int pre_off = 0;                              // set by the launcher: byte offset of that area
  unsigned long long* amax_out = nullptr;       // epilogue: per-row max |output| (atomicMax)
  unsigned long long* zero = nullptr; int nzero = 0;   // CTA 0 clears these words (for a later producer)
  unsigned long long* zero2 = nullptr; int nzero2 = 0; // a second range
  unsigned long long* nstat_out = nullptr;      // EPI_RESID: per row atomicMax max |x_new|, atomicAdd sum x_new^2
  int tail = TAIL_NONE;
  unsigned int* ticket = nullptr;
  const int64_t* tail_x = nullptr; int tail_ldx = 0; int tail_K = 0;
  const int64_t* tail_gain = nullptr;
  const unsigned long long* tail_amax = nullptr;
  const unsigned long long* tail_nstat = nullptr;   // TAIL_NORM: the row statistics (max |x|, sum x^2) the
                                                    // kernel's CTAs published (nstat_out), when given
  int16_t* tail_xq = nullptr; int tail_ldq = 0; int32_t* tail_xs = nullptr;
  AttnArgs rope;
  LinW L;
  int R = 1;
  int epi = EPI_STORE;
  int64_t* out = nullptr; int ldo = 0;
  int64_t* raw = nullptr; int ldr = 0;          // trace / raw output (row stride ldr)
  int64_t* raw2 = nullptr;                      // SwiGLU: raw of the up rows
  const int32_t* silu_t = nullptr;
  // Freivalds self-check, per LOGICAL linear ("segment") of a fused GEMV.  Segment rows of the
  // accumulator are (lhs_p1, lhs_p2, rhs_p1, rhs_p2), one row per activation row:
  //   lhs += sum_n r_p[n] * (tot_n mod P_p),   rhs += sum_k d_p[k] * (xq_k mod P_p)
  // RPU == 1: segment s covers fused columns [seg_start[s], seg_start[s] + seg_n[s]);
  // SwiGLU (RPU == 2): segment 0 = gate rows, segment 1 = up rows (local index = pair index).
  int fr_nseg = 0;
  int fr_seg_start[3] = {0, 0, 0};
  const int32_t* fr_r[3] = {nullptr, nullptr, nullptr};     // (2, n_seg) values in [0, P)
  const int32_t* fr_d[3] = {nullptr, nullptr, nullptr};     // (2, K)
  unsigned long long* fr_acc[3] = {nullptr, nullptr, nullptr};
  // greedy head
  unsigned long long* head_part = nullptr;      // (grid, R, 2) partial (value, index)
  unsigned int* head_ticket = nullptr;          // last-CTA counter
  int32_t* next_tok = nullptr;                  // (R)
  int64_t* head_val = nullptr;                  // (R) best value next to next_tok (tensor parallel)
  int* err = nullptr;
  int grid = 0;
  // tensor parallel (fused exchanges): tpx_in (XIN_QUANT) takes the row max over the ranks from
  // exchange TPX_AMAX_O / TPX_AMAX_H; tpx_out publishes this kernel's result as exchange tpx_out:
  // TPX_SUM_O / TPX_SUM_D (EPI_RAW: `raw` is this rank's own slot, the peers' slots are written
  // from the epilogue) or TPX_AMAX_H (the final amax_out rows, from the last CTA)
  const TpX* tpx = nullptr;                     // device memory
  int tpx_in = -1, tpx_out = -1;
  unsigned int* tpx_ticket = nullptr;
};

cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t st, bool pdl);
int gemv_grid(int N, bool swiglu);
cudaError_t launch_gemv_op(const int16_t* x16, const int8_t* wT, const int64_t* Mg, int K, int N, int64_t* out,
                           cudaStream_t st);

// One-shot tensor-parallel all-reduce over NVLink peer memory (tpcomm.cu)
constexpr int TPC_CH = 1024;                  // 8-byte elements per CTA slice
constexpr int TPC_MAX_RANKS = 8;
struct TpComm {
  int rank = 0, size = 1, nblk = 0;
  char* base[TPC_MAX_RANKS] = {};             // every rank's buffer, mapped into this process
  unsigned long long* epoch = nullptr;        // (nblk) this rank's call counters, one per slice
  int* err = nullptr;                         // device error word (wait timeout)
};
struct TpResid {                              // int64 SUM fused with the residual update
  int64_t* x = nullptr; int ldx = 0; int N = 0;
  const int32_t* xs = nullptr; const int64_t* b = nullptr;
  const unsigned long long* amax = nullptr;   // when set, the row shift is qrow_shift(amax[r]) (not xs)
  int64_t* tot = nullptr; int ldt = 0;        // optional copy of the full sums (trace)
};
// op 0: uint64 max, 1: int64 sum (with rz.x: x[r, j] += shr(sum, 28 - xs[r]) + b[j]), 2: int32 min,
// 3: int64 max
cudaError_t launch_tp_allreduce(const TpComm& c, const void* src, void* dst, int n, int op, const TpResid& rz,
                                cudaStream_t st, bool pdl = false);
// Consumer of TPX_SUM_O / TPX_SUM_D fused with the next norm: x[r] += shr(sum over ranks, 28 - s) + b with
// s = qrow_shift(max over ranks of TPX_AMAX_O / TPX_AMAX_H), then xq, xs = qrow(irms(x[r], g)).
cudaError_t launch_tpx_norm(const TpX& x, int sum_type, const int64_t* bias, int64_t* xr, int ldx, const int64_t* g,
                            int R, int D, int16_t* xq, int ldq, int32_t* xs, cudaStream_t st, bool pdl);
size_t tp_comm_bytes(int size, int nblk);

// tensor parallel helpers (rowops.cu)
// x[r, n] += shr(tot[r, n], 28 - xs[r]) (+ b[n]): the residual update after an all-reduced partial sum
// (amax given: the shift of row r is qrow_shift(amax[r]), the max the consumer GEMV's qrow used)
cudaError_t launch_tp_resid(const int64_t* tot, int R, int N, const int32_t* xs, const int64_t* b, int64_t* x, int ldx,
                            cudaStream_t st, const unsigned long long* amax = nullptr);
// next[r] = v0 + idx[r] when val[r] equals the all-reduced maximum gmax[r], else INT32_MAX (min-reduced next)
cudaError_t launch_tp_pick(const int64_t* val, const int64_t* gmax, int32_t* idx, int v0, int R, cudaStream_t st);

// per-row kernels
// nstat (optional): per row (max |x|, sum x^2) of the embedded row, for a XIN_NORMST consumer
cudaError_t launch_embed(const int8_t* emb, int emb_shift, const int32_t* ids, int R, int D, int64_t* x,
                         cudaStream_t st, bool pdl, unsigned long long* nstat = nullptr);
cudaError_t launch_embed64(const int64_t* emb_q16, const int32_t* ids, int R, int D, int64_t* x, cudaStream_t st,
                           bool pdl);
constexpr int TC_DECODE_ROWS = 8;
constexpr int TC_PAD_ROWS = 128;      // multi-row digit planes are padded to a multiple of this
// dig (optional): int8 digit planes of the rows for the tensor-core GEMM (planes of dig_rows rows)
// xcap (optional): a copy of each input row x (row stride ldcap), for the trace commitment
cudaError_t launch_norm_q(const int64_t* x, int ldx, const int64_t* g, int R, int D, int16_t* xq, int ldq,
                          int32_t* xs, cudaStream_t st, bool pdl, uint8_t* dig = nullptr, int64_t* xcap = nullptr,
                          int64_t ldcap = 0, int dig_rows = TC_DECODE_ROWS);

// ---- Merkle trace commitment (csrc/commit.cu)
struct CommitLayout {
  int NL = 0, D = 0, KV = 0, hd = 0;
  int64_t x_off = 0;                  // X[0..NL] (D each) within a log row
  int64_t kr_off = 0;                 // roped K | V of every layer (2 KV hd each)
  const int64_t* lin_off = nullptr;   // device: (7 NL + 1) accumulator offsets in the trace row
  const int64_t* lin_len = nullptr;   // device: their lengths
};
inline int64_t commit_leaf_count(int NL, int T) { return (int64_t)(5 * NL + 2) * T; }

// ---- weightless cell verifier (csrc/verify.cu)
struct VLinDev {                      // one logical linear, seen by the verifier (no weights)
  int N = 0, K = 0, group = 0;
  int row0 = 0, row_step = 1;         // its rows in the fused matrix (bias / per-channel scale index)
  int mbits = 0;                      // per channel: bitlen(max M) of the logical linear
  const int64_t* b = nullptr;         // fused bias or nullptr
  const int64_t* Mc = nullptr;        // fused per-channel scales (per-channel linears)
  const int32_t* r = nullptr;         // (2, N) Freivalds r
  const int32_t* d = nullptr;         // (2, K) Freivalds digests
};
struct VLeafRec {                     // one opened leaf of one cell
  int64_t voff = 0;                   // first value in the opened-values buffer
  int64_t leaf = 0;                   // index among the committed leaves
  int64_t poff = 0;                   // first proof byte
  int nseg = 0;
  int64_t len[4] = {0, 0, 0, 0};
};
enum Verdict {
  VERDICT_OK = 0, VERDICT_EMB = 2, VERDICT_KV = 3, VERDICT_KR = 4, VERDICT_Q = 5, VERDICT_O = 6,
  VERDICT_GU = 7, VERDICT_DOWN = 8, VERDICT_RESID = 9, VERDICT_HEAD = 10,
  VERDICT_MERKLE = 1000,              // + the position of the failing leaf among the cell's leaves
};
struct VerifyArgs {
  int NL = 0, D = 0, H = 0, KV = 0, hd = 0, I = 0, V = 0, T = 0;
  int64_t inv = 0;
  const VLinDev* lins = nullptr;      // 7 NL + 1
  const int64_t* const* g1 = nullptr; // device arrays of NL gain pointers
  const int64_t* const* g2 = nullptr;
  const int64_t* gf = nullptr;
  const int32_t *cos_t = nullptr, *sin_t = nullptr, *exp_t = nullptr, *silu_t = nullptr;
  const int32_t* emb_r = nullptr;     // (2, D)
  const int64_t* emb_de = nullptr;    // (2, V)
  const int32_t* ids = nullptr;       // (T)
  const int32_t* cells = nullptr;     // (n, 2): layer, position
  const int64_t* values = nullptr;    // opened values, cell after cell
  const int64_t* cell_voff = nullptr; // (n)
  const int* cell_leaf0 = nullptr;    // (n + 1): the cells' leaf records
  const int* leaf_ok = nullptr;
  int64_t* scratch = nullptr; int64_t scr_len = 0;
  int ymax = 0, q16_len = 0;
  int32_t* verdict = nullptr;
};
cudaError_t launch_verify(const VerifyArgs& a, int n_cells, int n_leaves, const VLeafRec* recs, const uint8_t* proofs,
                          int depth, const uint8_t* root, int* leaf_ok, cudaStream_t st);
cudaError_t launch_emb_digest(const int8_t* emb, int shift, const int64_t* emb_q16, int V, int D, const int32_t* r,
                              int64_t* de, cudaStream_t st);

// ---- integer sampler (csrc/sample.cu): token of each row, position pos[r] (advanced when pos_inc)
cudaError_t launch_sample(int R, const int64_t* logits, int V, int64_t ld, const unsigned long long* seeds, int32_t* pos,
                          bool pos_inc, int64_t tnum, const int32_t* exp_t, int32_t* tokens, cudaStream_t st, bool pdl);
cudaError_t launch_commit_log(int R, const int32_t* row_seq, const int32_t* row_pos, int seq, const int64_t* trace,
                              int64_t trace_row, const int64_t* cap, int64_t cap_row, int64_t* log, int npos_cap,
                              int* npos, int* err, cudaStream_t st);
cudaError_t commit_root(const int64_t* log, int64_t row, int T, const CommitLayout& c, uint8_t* leaves,
                        uint8_t* lv_a, uint8_t* lv_b, uint8_t** root_dev, cudaStream_t st);
cudaError_t launch_quant(const int64_t* x, int ldx, int R, int K, int16_t* xq, int ldq, int32_t* xs,
                         cudaStream_t st, bool pdl, uint8_t* dig = nullptr, int dig_rows = TC_DECODE_ROWS);
cudaError_t launch_quant_known(const int64_t* x, int ldx, int R, int K, const unsigned long long* amax, int16_t* xq,
                               int ldq, int32_t* xs, cudaStream_t st, bool pdl, uint8_t* dig = nullptr,
                               int dig_rows = TC_DECODE_ROWS);
cudaError_t launch_requant_channel(const int64_t* acc, int ld, int R, const LinW& L, int64_t* out, int ldo,
                                   const int32_t* xs, int epi, cudaStream_t st, bool pdl);

// per-channel head over many rows: requant of raw sums, optional logits, greedy next token per row
cudaError_t launch_head_rows(const int64_t* acc, int ld, int R, const LinW& L, const int32_t* xs, int64_t* logits,
                             int ldl, int32_t* next, cudaStream_t st);

cudaError_t launch_rope_cache(const AttnArgs& a, cudaStream_t st, bool pdl);
// attention; when xq_out is set, the last CTA also writes qrow(out) (shift from amax_out)
cudaError_t launch_attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_attn_rope(const AttnArgs& a, cudaStream_t st, bool pdl);   // decode rows, R <= 8
// prefill chunk of consecutive positions of one sequence (q rows and the K/V cache already written)
cudaError_t launch_attn_prefill(const AttnArgs& a, cudaStream_t st);
cudaError_t launch_embed_norm(const int8_t* emb, const int64_t* emb_q16, int emb_shift, const int32_t* ids, int R,
                              int D, const int64_t* g, int64_t* x, int16_t* xq, int ldq, int32_t* xs,
                              cudaStream_t st, bool pdl);

cudaError_t launch_fr_keys(const int8_t* w, const int32_t* Mg, int ldm, int N, int K, int row0, int row_step,
                           const int32_t* r, int32_t* d, cudaStream_t st);
cudaError_t launch_fr_check(const unsigned long long* acc, int nchecks, int* fail_count, int* err,
                            cudaStream_t st, bool pdl);

// ---------------------------------------------------------------- mixture of experts (moe.cu)
constexpr int MOE_MAX_EXPERTS = 128;
constexpr int MOE_MAX_TOPK = 8;

// One expert's per-channel SwiGLU MLP: gate|up rows interleaved (2j gate j, 2j+1 up j), (2I, D)
// int8 + int64 scales; down (D, I) + scales; bitlen of each logical linear's largest scale.
struct ExpertW {
  const int8_t* w_gu = nullptr;
  const int64_t* M_gu = nullptr;
  const int8_t* w_d = nullptr;
  const int64_t* M_d = nullptr;
  int I = 0;
  int mb_g = 0, mb_u = 0, mb_d = 0;
};

struct MoeArgs {
  int R = 0, D = 0, NE = 0, TOPK = 0, IMAX = 0;
  const int16_t* xq = nullptr; int ldq = 0; const int32_t* xs = nullptr;   // qrow(irms(x, g2)) rows
  const int8_t* w_router = nullptr; const int64_t* M_router = nullptr; int mbits_router = 0;
  const int8_t* w_sgate = nullptr; const int64_t* M_sgate = nullptr; int mbits_sgate = 0;
  const ExpertW* ex = nullptr;                 // NE + 1 entries; entry NE is the shared expert
  const int32_t* exp_t = nullptr; const int32_t* silu_t = nullptr; const int32_t* sig_t = nullptr;
  int32_t* sel = nullptr; int64_t* prob = nullptr; int64_t* sgv = nullptr;
  int32_t* sel_hist = nullptr;                 // optional copy of the selections (R, TOPK)
  int32_t* off = nullptr;                      // (NE + 2) slot offsets
  int32_t* slot_row = nullptr; int32_t* slot_exp = nullptr;   // (R * (TOPK + 1))
  int32_t* slot_of = nullptr;                  // (R * TOPK)
  int64_t* raw_gu = nullptr; int ld_gu = 0;    // (slots, 2 IMAX)
  int16_t* hq = nullptr; int ld_h = 0;         // (slots, IMAX)
  int32_t* hs = nullptr;                       // (slots)
  int64_t* raw_d = nullptr;                    // (slots, D)
};
// x[r] += MoE(m) for the R rows whose qrow(m) is in xq / xs
cudaError_t launch_moe(const MoeArgs& a, int64_t* x, int ldx, cudaStream_t st);

// ---------------------------------------------------------------- tcgen05 group-128 GEMM (many rows)
constexpr int TC_MIN_ROWS = 16;        // activation rows from which the tensor-core path is used
size_t gemm_tc_digit_bytes(int T, int K);
// int8 digit planes (lo = xq & 255, hi = xq >> 8) of T int16 rows, padded to the tile height
cudaError_t launch_digits(const int16_t* xq, int ldx, int T, int K, void* digits, cudaStream_t st);
bool gemm_tc_supported(const LinW& L, int epi);
void gemm_tc_set_persist(int on);     // multi-row GEMM on a persistent grid (default 1), process-wide
// Decode steps (T <= TC_DECODE_ROWS rows, digit planes of exactly TC_DECODE_ROWS rows): 8-row
// activation tiles, optional split over the 128-groups (int64 partial sums in tot_buf, the last
// CTA of each 128-row tile finishes it; tot_buf and tickets are zero between uses), SwiGLU row
// max published to amax_out, words cleared for a later producer, programmatic dependent launch.
struct TcDecode {
  int ksplit = 1;
  int64_t* tot_buf = nullptr;           // (TC_DECODE_ROWS, N) int64
  unsigned int* tickets = nullptr;      // (N / 128)
  unsigned long long* amax_out = nullptr;
  unsigned long long* zero = nullptr; int nzero = 0;
  bool pdl = false;
};
// tot / requant epilogue of a group-128 linear over T activation rows given as digit planes
cudaError_t launch_gemm_tc(const void* digits, int T, const LinW& L, const int32_t* xs, int epi, int64_t* out, int ldo,
                           int64_t* raw, int64_t* raw2, int ldr, const int32_t* silu_t, int* err, cudaStream_t st,
                           const TcDecode* dec = nullptr, unsigned long long* amax_out = nullptr);


}  // namespace exb
