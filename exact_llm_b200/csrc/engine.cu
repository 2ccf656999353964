// The exact integer model engine behind the C ABI (include/exactb200.h).
//
// Replaces the reference's torch engine (exact_torch.py TModel, experiments GraphDecoder and
// TLinG) with a native runtime: weights in one HBM arena in fused layouts (q|k|v rows
// concatenated, gate/up rows interleaved), a static KV cache (K int16 + int8 shift, V int32),
// CUDA-graph replay of each decode/prefill step (one graph per step shape, position and token
// read from device memory, as in GraphDecoder), on-device greedy feedback, trace capture written
// directly by the GEMV epilogues, and the Freivalds self-check accumulated inside the GEMVs.
#include <algorithm>
#include <cctype>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include <dlfcn.h>
#include <nccl.h>

#include "exactb200.h"
#include "common.cuh"
#include "exb_internal.h"

using namespace exb;

static thread_local std::string g_err;
void exb::set_last_error(const std::string& msg) { g_err = msg; }

#define FAIL(code, msg)     \
  do {                      \
    g_err = (msg);          \
    return (code);          \
  } while (0)
#define CK(call)                                                                    \
  do {                                                                              \
    cudaError_t e_ = (call);                                                        \
    if (e_ != cudaSuccess) {                                                        \
      g_err = std::string(#call) + " -> " + cudaGetErrorString(e_);                 \
      return EXB_ECUDA;                                                             \
    }                                                                               \
  } while (0)

static constexpr int RMAX = 4;          // activation rows per GEMV pass (CUDA-core decode path)
static constexpr int MOE_ROWS = 256;    // rows per MoE block call (the tensor-core chunk size)
static constexpr int SEL_CAP = 4096;    // rows of router selections kept for inspection
static constexpr int EXP_LEN_H = 256 * 40 + 2, SILU_LEN_H = 32 * 256 + 2;

static int bitlen_host(uint64_t v) { int b = 0; while (v) { ++b; v >>= 1; } return b; }

struct LinInfo {                        // one logical linear (reference naming) inside a fused matrix
  std::string name;
  int N = 0, K = 0;
  int Ng = 0, Kg = 0;                   // global shape (tensor parallel: this rank holds a slice)
  int r_lo = 0, c_lo = 0;               // global row / column of the slice's first element
  int row0 = 0, row_step = 1;           // its rows in the fused matrix
  LinW* fused = nullptr;                // owning fused matrix
  int trace_off = 0;
  int64_t g_off = 0;                    // offset in the global trace row (tensor parallel: all ranks' slices)
  bool col_split = false;               // tensor parallel: this rank holds output columns [r_lo, r_lo + N)
  bool kv_owner = true;                 // tensor parallel: this rank counts its k / v slice in the global key
  int mbits = 0;
  int32_t* fr_r = nullptr;              // (2, N)
  int32_t* fr_d = nullptr;              // (2, K)
  unsigned long long* fr_acc = nullptr; // (RMAX, 4)
};

struct LayerDev {
  int64_t* g1 = nullptr;
  int64_t* g2 = nullptr;
  LinW qkv, o, gu, down;
  int li[7];                            // q, k, v, o, gate, up, down -> index into lins
  // MoE layers (config 4): router, shared-expert gate, experts and the shared expert (index NE)
  LinW router, sgate;
  std::vector<LinW> exgu, exd;          // NE + 1 entries
  ExpertW* ex_dev = nullptr;            // device table (NE + 1)
};

struct exb_model {
  exb_config c{};
  bool group = true;
  bool finalized = false;
  bool pdl = true;
  bool trace_on = false, fr_on = false;
  int n_lin = 0;
  int Nqkv = 0, KMAX = 0, NMAX = 0;
  char* warena = nullptr; size_t wbytes = 0, woff = 0;
  char* rarena = nullptr; size_t rbytes = 0, roff = 0;
  int8_t* emb = nullptr; int64_t* emb_q16 = nullptr;
  int64_t* gf = nullptr;
  LinW head;
  std::vector<LayerDev> L;
  std::vector<LinInfo> lins;            // trace order
  int32_t *exp_t = nullptr, *silu_t = nullptr, *sig_t = nullptr, *cos_t = nullptr, *sin_t = nullptr;
  cudaStream_t st = nullptr;
  // runtime buffers
  int32_t *row_ids = nullptr, *row_seq = nullptr, *row_pos = nullptr;      // exb_forward rows (RMAX)
  int32_t *gen_ids = nullptr, *gen_seq = nullptr, *gen_pos = nullptr;      // generate rows (max_batch)
  int32_t* gen_step = nullptr; int32_t* gen_tokens = nullptr; int gen_cap = 0;
  int64_t *x = nullptr, *qkv = nullptr, *ao = nullptr, *hb = nullptr, *logits = nullptr, *rawb = nullptr;
  int16_t* xq = nullptr; int32_t* xs = nullptr;
  int16_t* qq = nullptr; int32_t* qs = nullptr;
  int32_t* next_tok = nullptr;
  unsigned long long *amax_o = nullptr, *amax_h = nullptr;   // per-row max |x| published by producers
  unsigned long long *nstat_a = nullptr, *nstat_b = nullptr; // per-row (max |x|, sum x^2) of the residual
                                                             // stream before norm1 / norm2 (fuse level 3)
  unsigned int* ticket = nullptr;                            // last-CTA election counter
  unsigned long long* head_part = nullptr; unsigned int* head_ticket = nullptr;
  int head_grid = 0;
  int sms = 148;
  int64_t* trace = nullptr; int64_t trace_row = 0;
  int64_t trace_row_g = 0;              // global trace row length (tensor parallel: every rank's slices)
  // Merkle trace commitment: per-row capture of X (NL+1 rows of D) and the roped K | V of every
  // layer (2 KV hd), appended with the trace row to a device log indexed by position
  bool commit_on = false; int commit_seq = 0; int commit_cap = 0;
  int64_t cap_row = 0;
  int64_t* cap = nullptr;               // (RMAX, cap_row), arena
  int* commit_npos = nullptr;           // device: 1 + the largest logged position, arena
  int64_t* commit_log = nullptr;        // (commit_cap, trace_row + cap_row), allocated by exb_commit_begin
  int64_t* commit_lin = nullptr;        // device: accumulator offsets | lengths in the trace row
  // integer sampler (exb_sampling): per-row seed and next sampling position, used by the decode
  // steps of exb_generate / exb_generate_device instead of the greedy argmax
  int step_kernels = 0;                 // kernel nodes of the last captured step graph
  bool samp_on = false, samp_active = false;
  int64_t samp_tnum = 1 << 16;
  unsigned long long* samp_seed = nullptr;   // (RMAX), arena
  int32_t* samp_pos = nullptr;               // (RMAX), arena
  // weightless verifier: embedding row digests (exb_verifier_emb_keys)
  int32_t* ver_emb_r = nullptr;              // (2, D)
  int64_t* ver_emb_de = nullptr;             // (2, V)
  unsigned long long* fr_acc = nullptr;
  int* fr_fail = nullptr; int* err = nullptr;
  int16_t* kc = nullptr; int8_t* ks = nullptr; int32_t* vc = nullptr;
  size_t kv_layer_elems = 0;           // B * KV * Smax * hd
  // host state
  std::vector<int> seq_len;
  std::vector<int64_t> trace_host; int64_t trace_rows = 0;
  int64_t fr_checks = 0;
  std::map<uint64_t, cudaGraphExec_t> graphs;
  int32_t *h_ids = nullptr, *h_seq = nullptr, *h_pos = nullptr;           // pinned staging
  // tensor parallel (tp > 1): this rank's slice of the model; cg = the global architecture
  exb_config cg{};
  int tp = 1, tp_rank = 0;
  int qh0 = 0, qh1 = 0, kh0 = 0, kh1 = 0, ig0 = 0, ig1 = 0, v0 = 0, v1 = 0, vmax = 0;
  ncclComm_t comm = nullptr;
  // one-shot peer-memory all-reduce (tpcomm.cu); NCCL when the peers cannot be mapped or "tpar" is 0
  TpComm tpc;
  bool tpc_on = false, tpar = true;
  char* tpc_local = nullptr;
  unsigned long long* tpc_epoch = nullptr;
  // fused exchanges (tpx.cuh) in the same mapped buffers, after the all-reduce area; "tpx" 0: the
  // all-reduce kernels instead
  TpX tpx;
  TpX* tpx_dev = nullptr;                   // the same description in device memory (kernel arguments)
  bool tpx_opt = true;
  unsigned long long* tpx_ep = nullptr;     // (4) exchange counters
  unsigned int* tpx_tickets = nullptr;      // (2) last-CTA tickets: attention, GEMVs
  int64_t* tp_tot = nullptr;                // (RMAX, D) partial sums of o / down
  int64_t* tp_hval = nullptr;               // (RMAX) shard best logit
  int64_t* tp_hmax = nullptr;               // (RMAX) all-reduced best logit
  int64_t* tp_gather = nullptr;             // (RMAX, tp, vmax) gathered logits
  // MoE runtime (rows up to MOE_ROWS per call of the block)
  int moe_imax = 0;
  int32_t *moe_sel = nullptr, *moe_off = nullptr, *moe_slot_row = nullptr, *moe_slot_exp = nullptr, *moe_slot_of = nullptr;
  int32_t *moe_hs = nullptr, *moe_hist = nullptr;   // hist: (NL, SEL_CAP, TOPK) router selections of the last call
  int64_t *moe_prob = nullptr, *moe_sgv = nullptr, *moe_raw_gu = nullptr, *moe_raw_d = nullptr;
  int16_t* moe_hq = nullptr;
  int64_t sel_rows = 0;                              // rows recorded in moe_hist by the last forward call
  // tensor-core prefill: buffers for chunks of up to pch rows (allocated on first use)
  int pch = 0;
  char* p_arena = nullptr;
  int32_t* p_rows = nullptr; int32_t* p_hrows = nullptr;            // device ids|seq|pos, pinned staging
  int64_t *p_x = nullptr, *p_qkv = nullptr, *p_ao = nullptr, *p_hb = nullptr, *p_raw = nullptr;
  int16_t *p_xq = nullptr, *p_qq = nullptr;
  int32_t *p_xs = nullptr, *p_qs = nullptr, *p_next = nullptr;
  void* p_dig = nullptr;
  unsigned long long* p_amax = nullptr;     // per-row max |h| published by the gate|up GEMM
  // persistent decode-step kernel (step.cu): per-layer descriptors and accumulators
  bool tc_on = true;                    // multi-row chunks on the tensor-core GEMM
  bool tail_norm = false;               // decode: the o and down GEMVs finish the next norm in their last CTA
  int fuse_in = 1;                      // GEMVs build their int16 input rows: 1 = qrow prologue (o, down),
                                        // 2 = also the norm (q|k|v, gate|up, head), 3 = the norm from the
                                        // row statistics the residual producers publish, 0 = separate kernels
  bool attn_fused = true;               // decode: RoPE + cache write inside the attention kernel
  bool attn_prefill = true;             // prefill chunks of one sequence: query-tile attention kernel
  bool tc_decode = false;               // decode-step linears on the tcgen05 GEMM (8-row tiles, split-K)
  uint8_t* dq = nullptr;                // digit planes of the decode rows (2 x TC_DECODE_ROWS x KMAX)
  int64_t* tc_tot = nullptr;            // split-K partial sums (TC_DECODE_ROWS x NMAX)
  unsigned int* tc_tickets = nullptr;   // split-K last-CTA counters (NMAX / 128)
};

// ------------------------------------------------------------------------------------------ helpers
template <typename T>
static T* walloc(exb_model* m, size_t n) {
  size_t off = (m->woff + 255) & ~size_t(255);
  m->woff = off + n * sizeof(T);
  return m->warena ? reinterpret_cast<T*>(m->warena + off) : nullptr;
}
template <typename T>
static T* ralloc(exb_model* m, size_t n) {
  size_t off = (m->roff + 255) & ~size_t(255);
  m->roff = off + n * sizeof(T);
  return m->rarena ? reinterpret_cast<T*>(m->rarena + off) : nullptr;
}

static void plan_weights(exb_model* m) {
  const exb_config& c = m->c;
  const int D = c.D, Hd = c.H * c.hd, I = c.I;
  m->woff = 0;
  m->L.assign(c.NL, LayerDev());
  auto mk = [&](LinW& W, int N, int K, bool bias) {
    W.N = N; W.K = K;
    W.w = walloc<int8_t>(m, (size_t)N * K);
    if (m->group) {
      W.ldm = ((K / 128) + 3) & ~3;          // scale rows padded to 16 bytes (bulk-copy alignment)
      W.Mg = walloc<int32_t>(m, (size_t)N * W.ldm);
    }
    else W.Mc = walloc<int64_t>(m, N);
    W.b = bias ? walloc<int64_t>(m, N) : nullptr;
  };
  for (int i = 0; i < c.NL; ++i) {
    LayerDev& Ld = m->L[i];
    Ld.g1 = walloc<int64_t>(m, D);
    Ld.g2 = walloc<int64_t>(m, D);
    mk(Ld.qkv, m->Nqkv, D, true);
    mk(Ld.o, D, Hd, false);
    if (c.n_experts) {
      mk(Ld.router, c.n_experts, D, false);
      mk(Ld.sgate, 1, D, false);
      Ld.exgu.assign(c.n_experts + 1, LinW());
      Ld.exd.assign(c.n_experts + 1, LinW());
      for (int e = 0; e <= c.n_experts; ++e) {
        const int Ie = e < c.n_experts ? c.moe_I : c.shared_I;
        mk(Ld.exgu[e], 2 * Ie, D, false);
        mk(Ld.exd[e], D, Ie, false);
      }
    } else {
      mk(Ld.gu, 2 * I, D, false);
      mk(Ld.down, D, I, false);
    }
  }
  m->emb = walloc<int8_t>(m, (size_t)m->cg.V * D);            // every rank embeds every token
  m->gf = walloc<int64_t>(m, D);
  m->head.N = c.V; m->head.K = D;
  m->head.w = c.tie ? (m->emb ? m->emb + (size_t)m->v0 * D : nullptr) : walloc<int8_t>(m, (size_t)c.V * D);
  m->head.Mc = walloc<int64_t>(m, c.V);
  m->exp_t = walloc<int32_t>(m, EXP_LEN_H);
  m->silu_t = walloc<int32_t>(m, SILU_LEN_H);
  m->sig_t = walloc<int32_t>(m, SILU_LEN_H);
  m->cos_t = walloc<int32_t>(m, (size_t)c.rope_len * (c.hd / 2));
  m->sin_t = walloc<int32_t>(m, (size_t)c.rope_len * (c.hd / 2));
}

static void plan_lins(exb_model* m) {
  const exb_config& c = m->c;
  m->lins.clear();
  int off = 0;
  auto add = [&](const std::string& nm, LinW* f, int N, int K, int row0, int step) {
    LinInfo li; li.name = nm; li.N = N; li.K = K; li.row0 = row0; li.row_step = step; li.fused = f;
    li.Ng = N; li.Kg = K;
    li.trace_off = off; off += N;
    m->lins.push_back(li);
    return (int)m->lins.size() - 1;
  };
  const int qn = c.H * c.hd, kn = c.KV * c.hd;
  for (int i = 0; i < c.NL; ++i) {
    LayerDev& Ld = m->L[i];
    std::string p = "L" + std::to_string(i) + ".";
    Ld.li[0] = add(p + "q", &Ld.qkv, qn, c.D, 0, 1);
    Ld.li[1] = add(p + "k", &Ld.qkv, kn, c.D, qn, 1);
    Ld.li[2] = add(p + "v", &Ld.qkv, kn, c.D, qn + kn, 1);
    Ld.li[3] = add(p + "o", &Ld.o, c.D, qn, 0, 1);
    if (c.n_experts) {
      const int NE = c.n_experts;
      add(p + "router", &Ld.router, NE, c.D, 0, 1);
      add(p + "sgate", &Ld.sgate, 1, c.D, 0, 1);
      add(p + "sg", &Ld.exgu[NE], c.shared_I, c.D, 0, 2);
      add(p + "su", &Ld.exgu[NE], c.shared_I, c.D, 1, 2);
      add(p + "sd", &Ld.exd[NE], c.D, c.shared_I, 0, 1);
      for (int e = 0; e < NE; ++e) {
        const std::string q = p + "e" + std::to_string(e) + ".";
        add(q + "g", &Ld.exgu[e], c.moe_I, c.D, 0, 2);
        add(q + "u", &Ld.exgu[e], c.moe_I, c.D, 1, 2);
        add(q + "d", &Ld.exd[e], c.D, c.moe_I, 0, 1);
      }
      Ld.li[4] = Ld.li[5] = Ld.li[6] = -1;
      continue;
    }
    Ld.li[4] = add(p + "gate", &Ld.gu, c.I, c.D, 0, 2);
    Ld.li[5] = add(p + "up", &Ld.gu, c.I, c.D, 1, 2);
    Ld.li[6] = add(p + "down", &Ld.down, c.D, c.I, 0, 1);
  }
  add("head", &m->head, c.V, c.D, 0, 1);
  m->n_lin = (int)m->lins.size();
  if (m->tp > 1) {
    // global shapes and slice offsets of this rank (column-split q/k/v, gate/up, head; row-split o, down)
    const exb_config& g = m->cg;
    const int mm = (m->tp % g.KV == 0) ? m->tp / g.KV : 1;   // ranks sharing one KV head
    for (auto& L : m->lins) {
      const std::string t = L.name.substr(L.name.find('.') + 1);
      if (L.name == "head") { L.Ng = g.V; L.r_lo = m->v0; L.col_split = true; continue; }
      if (t == "q") { L.Ng = g.H * g.hd; L.r_lo = m->qh0 * g.hd; L.col_split = true; }
      else if (t == "k" || t == "v") {
        L.Ng = g.KV * g.hd; L.r_lo = m->kh0 * g.hd; L.col_split = true; L.kv_owner = m->tp_rank % mm == 0;
      }
      else if (t == "o") { L.Kg = g.H * g.hd; L.c_lo = m->qh0 * g.hd; }
      else if (t == "gate" || t == "up") { L.Ng = g.I; L.r_lo = m->ig0 * 128; L.col_split = true; }
      else if (t == "down") { L.Kg = g.I; L.c_lo = m->ig0 * 128; }
    }
  }
  int64_t goff = 0;
  for (auto& L : m->lins) { L.g_off = goff; goff += L.Ng; }
  m->trace_row_g = goff;
  m->trace_row = off;
}

static void plan_runtime(exb_model* m) {
  const exb_config& c = m->c;
  m->roff = 0;
  m->row_ids = ralloc<int32_t>(m, 3 * RMAX);              // ids | seq | pos, one block (one H2D copy)
  m->row_seq = m->row_ids ? m->row_ids + RMAX : nullptr;
  m->row_pos = m->row_ids ? m->row_ids + 2 * RMAX : nullptr;
  m->gen_ids = ralloc<int32_t>(m, c.max_batch); m->gen_seq = ralloc<int32_t>(m, c.max_batch);
  m->gen_pos = ralloc<int32_t>(m, c.max_batch); m->gen_step = ralloc<int32_t>(m, 1);
  m->x = ralloc<int64_t>(m, (size_t)RMAX * c.D);
  m->xq = ralloc<int16_t>(m, (size_t)RMAX * m->KMAX);
  m->xs = ralloc<int32_t>(m, RMAX);
  m->qkv = ralloc<int64_t>(m, (size_t)RMAX * m->Nqkv);
  m->qq = ralloc<int16_t>(m, (size_t)RMAX * c.H * c.hd);
  m->qs = ralloc<int32_t>(m, (size_t)RMAX * c.H);
  m->ao = ralloc<int64_t>(m, (size_t)RMAX * c.H * c.hd);
  m->hb = ralloc<int64_t>(m, (size_t)RMAX * c.I);
  m->logits = ralloc<int64_t>(m, (size_t)RMAX * std::max(c.V, m->vmax));
  m->rawb = ralloc<int64_t>(m, (size_t)RMAX * m->NMAX);
  m->next_tok = ralloc<int32_t>(m, RMAX);
  m->amax_o = ralloc<unsigned long long>(m, RMAX);
  m->amax_h = ralloc<unsigned long long>(m, RMAX);
  m->nstat_a = ralloc<unsigned long long>(m, 2 * RMAX);
  m->nstat_b = ralloc<unsigned long long>(m, 2 * RMAX);
  m->ticket = ralloc<unsigned int>(m, 4);
  m->head_part = ralloc<unsigned long long>(m, (size_t)m->head_grid * RMAX * 2);
  m->head_ticket = ralloc<unsigned int>(m, 1);
  m->trace = ralloc<int64_t>(m, (size_t)RMAX * m->trace_row);
  m->cap_row = (int64_t)(c.NL + 1) * c.D + (int64_t)c.NL * 2 * c.KV * c.hd;
  m->cap = ralloc<int64_t>(m, (size_t)RMAX * m->cap_row);
  m->commit_npos = ralloc<int>(m, 1);
  m->samp_seed = ralloc<unsigned long long>(m, RMAX);
  m->samp_pos = ralloc<int32_t>(m, RMAX);
  m->fr_acc = ralloc<unsigned long long>(m, (size_t)m->n_lin * RMAX * 4);
  m->fr_fail = ralloc<int>(m, 1);
  m->err = ralloc<int>(m, 1);
  m->kv_layer_elems = (size_t)c.max_batch * c.KV * c.max_seq * c.hd;
  m->kc = ralloc<int16_t>(m, m->kv_layer_elems * c.NL);
  m->vc = ralloc<int32_t>(m, m->kv_layer_elems * c.NL);
  m->ks = ralloc<int8_t>(m, (size_t)c.max_batch * c.KV * c.max_seq * c.NL);
  if (c.n_experts) {
    const int NE = c.n_experts, TK = c.topk, slots = MOE_ROWS * (TK + 1);
    m->moe_imax = std::max(c.moe_I, c.shared_I);
    m->moe_sel = ralloc<int32_t>(m, (size_t)MOE_ROWS * TK);
    m->moe_prob = ralloc<int64_t>(m, (size_t)MOE_ROWS * TK);
    m->moe_sgv = ralloc<int64_t>(m, MOE_ROWS);
    m->moe_off = ralloc<int32_t>(m, NE + 2);
    m->moe_slot_row = ralloc<int32_t>(m, slots);
    m->moe_slot_exp = ralloc<int32_t>(m, slots);
    m->moe_slot_of = ralloc<int32_t>(m, (size_t)MOE_ROWS * TK);
    m->moe_raw_gu = ralloc<int64_t>(m, (size_t)slots * 2 * m->moe_imax);
    m->moe_hq = ralloc<int16_t>(m, (size_t)slots * m->moe_imax);
    m->moe_hs = ralloc<int32_t>(m, slots);
    m->moe_raw_d = ralloc<int64_t>(m, (size_t)slots * c.D);
    m->moe_hist = ralloc<int32_t>(m, (size_t)c.NL * SEL_CAP * TK);
    for (int i = 0; i < c.NL; ++i) m->L[i].ex_dev = ralloc<ExpertW>(m, NE + 1);
  }
  if (m->tp > 1) {
    m->tp_tot = ralloc<int64_t>(m, (size_t)RMAX * c.D);
    m->tp_hval = ralloc<int64_t>(m, RMAX);
    m->tp_hmax = ralloc<int64_t>(m, RMAX);
    m->tp_gather = ralloc<int64_t>(m, (size_t)RMAX * m->tp * m->vmax);
  }
  m->dq = ralloc<uint8_t>(m, (size_t)2 * TC_DECODE_ROWS * m->KMAX);
  m->tc_tot = ralloc<int64_t>(m, (size_t)TC_DECODE_ROWS * m->NMAX);
  m->tc_tickets = ralloc<unsigned int>(m, m->NMAX / 128 + 1);
}

// ------------------------------------------------------------------------------------------ step
// One forward pass of R (<= RMAX) rows through every layer and the head.  Rows read their token,
// sequence slot and position from device arrays, so the enqueued work is identical for every
// step and can be captured once into a CUDA graph.
static std::vector<cudaEvent_t>* g_prof = nullptr;   // profiling: an event after every launch

// NCCL is resolved at run time, on the first tensor-parallel call, so that a process which loads
// this library before torch still gets torch's own NCCL: the copy already in the process is used
// when there is one (torch imports it), else the system libnccl.so.2.
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
};
static const NcclApi* nccl() {
  static NcclApi api;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h) {
      api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
      api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(h, "ncclCommInitRank");
      api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
      api.all_reduce = (decltype(api.all_reduce))dlsym(h, "ncclAllReduce");
      api.all_gather = (decltype(api.all_gather))dlsym(h, "ncclAllGather");
    }
  }
  return (api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce && api.all_gather) ? &api
                                                                                                          : nullptr;
}

// NCCL all-reduce on the model stream (captured into the step graph like any kernel)
static cudaError_t tp_allreduce(exb_model* m, const void* src, void* dst, size_t n, ncclDataType_t t, ncclRedOp_t op,
                                cudaStream_t st) {
  return nccl()->all_reduce(src, dst, n, t, op, m->comm, st) == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

// MoE block arguments for layer i over R rows (qrow(m) rows xq / xs); selections recorded at row
// hist_row0 of the layer's history when hist_row0 >= 0
static MoeArgs moe_args(exb_model* m, int i, int R, const int16_t* xq, int ldq, const int32_t* xs, int hist_row0) {
  const exb_config& c = m->c;
  LayerDev& Ld = m->L[i];
  MoeArgs a;
  a.R = R; a.D = c.D; a.NE = c.n_experts; a.TOPK = c.topk; a.IMAX = m->moe_imax;
  a.xq = xq; a.ldq = ldq; a.xs = xs;
  a.w_router = Ld.router.w; a.M_router = Ld.router.Mc; a.mbits_router = Ld.router.mbits;
  a.w_sgate = Ld.sgate.w; a.M_sgate = Ld.sgate.Mc; a.mbits_sgate = Ld.sgate.mbits;
  a.ex = Ld.ex_dev;
  a.exp_t = m->exp_t; a.silu_t = m->silu_t; a.sig_t = m->sig_t;
  a.sel = m->moe_sel; a.prob = m->moe_prob; a.sgv = m->moe_sgv;
  a.sel_hist = (hist_row0 >= 0 && hist_row0 + R <= SEL_CAP) ? m->moe_hist + ((size_t)i * SEL_CAP + hist_row0) * c.topk
                                                              : nullptr;
  a.off = m->moe_off; a.slot_row = m->moe_slot_row; a.slot_exp = m->moe_slot_exp; a.slot_of = m->moe_slot_of;
  a.raw_gu = m->moe_raw_gu; a.ld_gu = 2 * m->moe_imax; a.hq = m->moe_hq; a.ld_h = m->moe_imax; a.hs = m->moe_hs;
  a.raw_d = m->moe_raw_d;
  return a;
}
static int g_hist_row0 = -1;                             // selection-history row of the step being enqueued

static cudaError_t enqueue_step(exb_model* m, int R, const int32_t* ids, const int32_t* seq, const int32_t* pos,
                                bool want_logits, cudaStream_t st) {
  const exb_config& c = m->c;
  const bool pdl = m->pdl && !g_prof;
  const bool tp = m->tp > 1;
  const bool cm = m->commit_on;        // trace commitment capture (implies trace capture)
  const bool smp = m->samp_active;     // the next tokens come from the integer sampler
  const bool tcd = m->tc_decode && m->group && !m->trace_on && !m->fr_on && !tp && !c.n_experts && R <= TC_DECODE_ROWS &&
                   gemm_tc_supported(m->L[0].qkv, EPI_STORE) && gemm_tc_supported(m->L[0].o, EPI_RESID) &&
                   gemm_tc_supported(m->L[0].gu, EPI_SWIGLU) && gemm_tc_supported(m->L[0].down, EPI_RESID);
  cudaError_t e;
#define RUN(x)                                                    \
  do {                                                            \
    e = (x);                                                      \
    if (e != cudaSuccess) return e;                               \
    if (g_prof) {                                                 \
      cudaEvent_t ev;                                             \
      cudaEventCreate(&ev);                                       \
      cudaEventRecord(ev, st);                                    \
      g_prof->push_back(ev);                                      \
    }                                                             \
  } while (0)
  if (m->fr_on) RUN(cudaMemsetAsync(m->fr_acc, 0, sizeof(unsigned long long) * m->n_lin * RMAX * 4, st));
  // norm from published row statistics (fuse level 3): dense single-GPU models without capture
  const bool fzs = m->fuse_in >= 3 && !m->fr_on && !cm && !tp && !c.n_experts && !m->emb_q16 && !tcd;
  // norms as the last-CTA tails of the o and down GEMVs, from the row statistics their CTAs publish
  // (the embedding kernel norms layer 0's input): no norm kernels
  const bool ftail = m->tail_norm && m->fuse_in == 1 && !m->fr_on && !cm && !tp && !c.n_experts && !tcd;
  if (ftail)
    RUN(launch_embed_norm(m->emb_q16 ? nullptr : m->emb, m->emb_q16, c.emb_shift, ids, R, c.D, m->L[0].g1, m->x,
                          m->xq, m->KMAX, m->xs, st, false));
  else if (m->emb_q16) RUN(launch_embed64(m->emb_q16, ids, R, c.D, m->x, st, false));   // general Q16 rows
  else RUN(launch_embed(m->emb, c.emb_shift, ids, R, c.D, m->x, st, false,               // int8 rows << shift
                        fzs ? m->nstat_a : nullptr));
  const int Hd = c.H * c.hd;
  AttnArgs aa;
  aa.qkv = m->qkv; aa.ldqkv = m->Nqkv; aa.row_seq = seq; aa.row_pos = pos;
  aa.cos_t = m->cos_t; aa.sin_t = m->sin_t; aa.qq = m->qq; aa.qs = m->qs; aa.exp_t = m->exp_t;
  aa.out = m->ao; aa.ldo = Hd; aa.R = R; aa.H = c.H; aa.KV = c.KV; aa.hd = c.hd; aa.Smax = c.max_seq;
  aa.Tmax = c.rope_len; aa.err = m->err;
  // INV = round(2^16 / sqrt(hd)) (exact_llm.py:164): correctly rounded sqrt and division, ties to even
  aa.inv = (int64_t)std::nearbyint(65536.0 / std::sqrt((double)c.hd));
  auto trace_ptr = [&](int li) -> int64_t* { return m->trace_on ? m->trace + m->lins[li].trace_off : nullptr; };
  // tensor-parallel all-reduces: the one-shot peer-memory kernel, else NCCL (both inside the graph)
  const bool tpc = tp && m->tpc_on && m->tpar;
  // fused exchanges: no all-reduce kernels in the layers (the producers write into the peers' memory,
  // the consumers wait for their flags); the trace / Freivalds / commitment captures keep the
  // all-reduce kernels, which also give them the full sums
  const bool tpf = tpc && m->tpx_opt && m->fuse_in == 1 && m->attn_fused && !m->trace_on && !m->fr_on && !cm &&
                   !c.n_experts;
  // this rank's own partial-sum slot of a row-split linear (which 0: o, 1: down)
  auto own_slot = [&](int which) {
    return reinterpret_cast<int64_t*>(m->tpx.base[m->tp_rank]) + (size_t)2 * m->tp * TPX_ROWS +
           ((size_t)which * m->tp + m->tp_rank) * TPX_ROWS * c.D;
  };
  auto ar = [&](const void* src, void* dst, size_t n, ncclDataType_t t, ncclRedOp_t op, int myop) -> cudaError_t {
    if (tpc) return launch_tp_allreduce(m->tpc, src, dst, (int)n, myop, TpResid(), st, pdl);
    return tp_allreduce(m, src, dst, n, t, op, st);
  };
  // SUM of a row-split linear's partial sums, then x += shr(tot, 28 - s) + b (and the trace copy);
  // s = the shift of the linear's input row: from the all-reduced max when its GEMV built the row
  // in its prologue (amax given), else the one the separate qrow kernel wrote to m->xs
  auto ar_resid = [&](const int64_t* bias, int64_t* trace_dst, const unsigned long long* amax) -> cudaError_t {
    if (tpc) {
      TpResid rz;
      rz.x = m->x; rz.ldx = c.D; rz.N = c.D; rz.xs = m->xs; rz.b = bias; rz.amax = amax;
      rz.tot = trace_dst; rz.ldt = (int)m->trace_row;
      return launch_tp_allreduce(m->tpc, m->tp_tot, nullptr, R * c.D, 1, rz, st, pdl);
    }
    cudaError_t e2 = tp_allreduce(m, m->tp_tot, m->tp_tot, (size_t)R * c.D, ncclInt64, ncclSum, st);
    if (e2 == cudaSuccess && trace_dst)
      e2 = cudaMemcpy2DAsync(trace_dst, sizeof(int64_t) * m->trace_row, m->tp_tot, sizeof(int64_t) * c.D,
                             sizeof(int64_t) * c.D, R, cudaMemcpyDeviceToDevice, st);
    if (e2 == cudaSuccess) e2 = launch_tp_resid(m->tp_tot, R, c.D, m->xs, bias, m->x, c.D, st, amax);
    return e2;
  };
  auto set_fr = [&](GemvArgs& g, std::initializer_list<int> lis, int nseg_start_override = -1) {
    (void)nseg_start_override;
    if (!m->fr_on) return;
    int s = 0;
    for (int li : lis) {
      const LinInfo& L = m->lins[li];
      g.fr_seg_start[s] = L.row_step == 1 ? L.row0 : 0;
      g.fr_r[s] = L.fr_r;
      g.fr_d[s] = L.fr_d;
      g.fr_acc[s] = L.fr_acc;
      ++s;
    }
    g.fr_nseg = s;
  };
  // Per layer (every kernel chained with programmatic dependent launch, so each GEMV is resident
  // and pulling its weights into L2 while the small kernel before it runs):
  //   norm          xq, s = qrow(irms(x, g1))               (one CTA per row)
  //   q|k|v GEMV    -> q|k|v rows
  //   rope/cache    RoPE, K/V cache write, quantised query rows
  //   attention     cluster per (row, KV head); publishes max |out| per row
  //   quant         xq = qrow(out) with the published max   (row split over CTAs)
  //   o GEMV        x += o(...)
  //   norm          xq, s = qrow(irms(x, g2))
  //   gate|up GEMV  h = shr(isilu(g)*u, 16); publishes max |h| per row
  //   quant         xq = qrow(h)
  //   down GEMV     x += down(h)
  aa.amax_out = m->amax_o;
  if (tpf) { aa.tpx = m->tpx_dev; aa.tpx_ticket = m->tpx_tickets; }
  for (int i = 0; i < c.NL; ++i) {
    LayerDev& Ld = m->L[i];
    const size_t kvoff = m->kv_layer_elems * i;
    aa.kc = m->kc + kvoff; aa.vc = m->vc + kvoff;
    aa.ks = m->ks + (size_t)c.max_batch * c.KV * c.max_seq * i;
    auto base = [&](GemvArgs& g, const LinW& L) {
      g.L = L; g.R = R; g.err = m->err; g.ldr = (int)m->trace_row;
      g.xq = m->xq; g.xs = m->xs; g.ldx = m->KMAX;
    };
    if (tcd) {
      // tensor-core decode: the row kernels also write the int8 digit planes the GEMM reads; the
      // narrow matrices split their 128-groups over more CTAs (int64 partial sums, last CTA finishes)
      auto dec = [&](const LinW& L) {
        TcDecode d;
        const int tiles = L.N / 128, G = L.K / 128;
        d.ksplit = std::max(1, std::min(G, (2 * m->sms + tiles - 1) / tiles));
        d.tot_buf = m->tc_tot; d.tickets = m->tc_tickets; d.pdl = pdl;
        return d;
      };
      RUN(launch_norm_q(m->x, c.D, Ld.g1, R, c.D, m->xq, m->KMAX, m->xs, st, pdl, m->dq));
      {
        TcDecode d = dec(Ld.qkv);
        d.zero = m->amax_o; d.nzero = RMAX;
        RUN(launch_gemm_tc(m->dq, R, Ld.qkv, m->xs, EPI_STORE, m->qkv, m->Nqkv, nullptr, nullptr, 0, nullptr, m->err,
                           st, &d));
      }
      if (m->attn_fused) {
        RUN(launch_attn_rope(aa, st, pdl));
      } else {
        RUN(launch_rope_cache(aa, st, pdl));
        RUN(launch_attn_decode(aa, st, pdl));
      }
      RUN(launch_quant_known(m->ao, Hd, R, Hd, m->amax_o, m->xq, m->KMAX, m->xs, st, pdl, m->dq));
      {
        TcDecode d = dec(Ld.o);
        d.zero = m->amax_h; d.nzero = RMAX;
        RUN(launch_gemm_tc(m->dq, R, Ld.o, m->xs, EPI_RESID, m->x, c.D, nullptr, nullptr, 0, nullptr, m->err, st, &d));
      }
      RUN(launch_norm_q(m->x, c.D, Ld.g2, R, c.D, m->xq, m->KMAX, m->xs, st, pdl, m->dq));
      {
        TcDecode d = dec(Ld.gu);
        d.amax_out = m->amax_h;
        RUN(launch_gemm_tc(m->dq, R, Ld.gu, m->xs, EPI_SWIGLU, m->hb, c.I, nullptr, nullptr, 0, m->silu_t, m->err, st,
                           &d));
      }
      RUN(launch_quant_known(m->hb, c.I, R, c.I, m->amax_h, m->xq, m->KMAX, m->xs, st, pdl, m->dq));
      {
        TcDecode d = dec(Ld.down);
        RUN(launch_gemm_tc(m->dq, R, Ld.down, m->xs, EPI_RESID, m->x, c.D, nullptr, nullptr, 0, nullptr, m->err, st,
                           &d));
      }
      continue;
    }
    // fused inputs: each GEMV CTA computes its int16 rows in its prologue (qrow with the
    // producer's published max at level 1, also the norm at level 2) while its first weight bytes
    // stream into L2
    // o and down: qrow in the prologue from the producer's published (under tensor parallelism:
    // all-reduced) row max; the residual update after the all-reduce derives the shift from it
    const bool fz = m->fuse_in >= 1 && !m->fr_on;
    const bool fzn = m->fuse_in == 2 && !m->fr_on && !cm;  // q|k|v and gate|up: norm in the prologue
    if (tpf && i > 0)   // the previous layer's down exchange, residual update and this norm
      RUN(launch_tpx_norm(m->tpx, TPX_SUM_D, m->L[i - 1].down.b, m->x, c.D, Ld.g1, R, c.D, m->xq, m->KMAX, m->xs, st,
                          pdl));
    else if (!fzn && !fzs && !ftail)
      RUN(launch_norm_q(m->x, c.D, Ld.g1, R, c.D, m->xq, m->KMAX, m->xs, st, pdl, nullptr,
                        cm ? m->cap + (size_t)i * c.D : nullptr, m->cap_row));
    {
      GemvArgs g; base(g, Ld.qkv);
      if (fzn) { g.xin = XIN_NORM; g.x64 = m->x; g.ldx64 = c.D; g.gain = Ld.g1; }
      if (fzs) { g.xin = XIN_NORMST; g.x64 = m->x; g.ldx64 = c.D; g.gain = Ld.g1; g.nstat_in = m->nstat_a; }
      g.epi = EPI_STORE; g.out = m->qkv; g.ldo = m->Nqkv; g.raw = trace_ptr(Ld.li[0]);
      g.zero = m->amax_o; g.nzero = RMAX;
      if (fzs || ftail) { g.zero2 = m->nstat_b; g.nzero2 = 2 * RMAX; }   // o accumulates norm2's statistics
      set_fr(g, {Ld.li[0], Ld.li[1], Ld.li[2]});
      RUN(launch_gemv(g, st, pdl));
    }
    if (m->attn_fused || cm) {
      aa.kr_out = cm ? m->cap + (size_t)(c.NL + 1) * c.D + (size_t)i * 2 * c.KV * c.hd : nullptr;
      aa.ldkr = m->cap_row;
      RUN(launch_attn_rope(aa, st, pdl));
    } else {
      RUN(launch_rope_cache(aa, st, pdl));
      RUN(launch_attn_decode(aa, st, pdl));
    }
    // tensor parallel: the qrow of o's input needs the max over every rank's heads
    if (tp && !tpf) RUN(ar(m->amax_o, m->amax_o, R, ncclUint64, ncclMax, 0));
    if (!fz) RUN(launch_quant_known(m->ao, Hd, R, Hd, m->amax_o, m->xq, m->KMAX, m->xs, st, pdl && !tp));
    {
      GemvArgs g; base(g, Ld.o);
      if (fz) { g.xin = XIN_QUANT; g.x64 = m->ao; g.ldx64 = Hd; g.amax_in = m->amax_o; }
      g.epi = EPI_RESID; g.out = m->x; g.ldo = c.D; g.raw = trace_ptr(Ld.li[3]);
      g.zero = m->amax_h; g.nzero = RMAX;
      if (fzs || ftail) g.nstat_out = m->nstat_b;
      if (ftail) {   // norm2 in the last CTA: xq, s = qrow(irms(x, g2)) for the gate|up GEMV
        g.tail = TAIL_NORM; g.ticket = m->ticket; g.tail_x = m->x; g.tail_ldx = c.D; g.tail_K = c.D;
        g.tail_gain = Ld.g2; g.tail_nstat = m->nstat_b; g.tail_xq = m->xq; g.tail_ldq = m->KMAX; g.tail_xs = m->xs;
      }
      if (tp) { g.epi = EPI_RAW; g.out = nullptr; g.raw = m->tp_tot; g.ldr = c.D; }   // partial sums over own heads
      if (tpf) {
        g.tpx = m->tpx_dev; g.tpx_in = TPX_AMAX_O; g.tpx_out = TPX_SUM_O; g.tpx_ticket = m->tpx_tickets + 1;
        g.raw = own_slot(0);
      }
      set_fr(g, {Ld.li[3]});
      RUN(launch_gemv(g, st, pdl));
    }
    if (tp && !tpf) RUN(ar_resid(Ld.o.b, trace_ptr(Ld.li[3]), fz ? m->amax_o : nullptr));   // trace: o's full sum
    if (tpf)
      RUN(launch_tpx_norm(m->tpx, TPX_SUM_O, Ld.o.b, m->x, c.D, Ld.g2, R, c.D, m->xq, m->KMAX, m->xs, st, pdl));
    else if ((!fzn && !fzs && !ftail) || c.n_experts)
      RUN(launch_norm_q(m->x, c.D, Ld.g2, R, c.D, m->xq, m->KMAX, m->xs, st, pdl));
    if (c.n_experts) {
      RUN(launch_moe(moe_args(m, i, R, m->xq, m->KMAX, m->xs, g_hist_row0), m->x, c.D, st));
      continue;
    }
    {
      GemvArgs g; base(g, Ld.gu);
      if (fzn) { g.xin = XIN_NORM; g.x64 = m->x; g.ldx64 = c.D; g.gain = Ld.g2; }
      if (fzs) {
        g.xin = XIN_NORMST; g.x64 = m->x; g.ldx64 = c.D; g.gain = Ld.g2; g.nstat_in = m->nstat_b;
        g.zero2 = m->nstat_a; g.nzero2 = 2 * RMAX;                       // down accumulates the next norm1's
      }
      if (ftail) { g.zero2 = m->nstat_a; g.nzero2 = 2 * RMAX; }
      g.epi = EPI_SWIGLU; g.out = m->hb; g.ldo = c.I; g.silu_t = m->silu_t; g.amax_out = m->amax_h;
      g.raw = trace_ptr(Ld.li[4]); g.raw2 = trace_ptr(Ld.li[5]);
      if (tpf) { g.tpx = m->tpx_dev; g.tpx_out = TPX_AMAX_H; g.tpx_ticket = m->tpx_tickets + 1; }
      set_fr(g, {Ld.li[4], Ld.li[5]});
      RUN(launch_gemv(g, st, pdl));
    }
    if (tp && !tpf) RUN(ar(m->amax_h, m->amax_h, R, ncclUint64, ncclMax, 0));
    if (!fz) RUN(launch_quant_known(m->hb, c.I, R, c.I, m->amax_h, m->xq, m->KMAX, m->xs, st, pdl && !tp));
    {
      GemvArgs g; base(g, Ld.down);
      if (fz) { g.xin = XIN_QUANT; g.x64 = m->hb; g.ldx64 = c.I; g.amax_in = m->amax_h; }
      g.epi = EPI_RESID; g.out = m->x; g.ldo = c.D; g.raw = trace_ptr(Ld.li[6]);
      if (fzs || ftail) g.nstat_out = m->nstat_a;
      if (ftail) {   // the next layer's norm1 (or the final norm) in the last CTA
        g.tail = TAIL_NORM; g.ticket = m->ticket; g.tail_x = m->x; g.tail_ldx = c.D; g.tail_K = c.D;
        g.tail_gain = i + 1 < c.NL ? m->L[i + 1].g1 : m->gf; g.tail_nstat = m->nstat_a;
        g.tail_xq = m->xq; g.tail_ldq = m->KMAX; g.tail_xs = m->xs;
      }
      if (tp) { g.epi = EPI_RAW; g.out = nullptr; g.raw = m->tp_tot; g.ldr = c.D; }   // partial sums over own groups
      if (tpf) {
        g.tpx = m->tpx_dev; g.tpx_in = TPX_AMAX_H; g.tpx_out = TPX_SUM_D; g.tpx_ticket = m->tpx_tickets + 1;
        g.raw = own_slot(1);
      }
      set_fr(g, {Ld.li[6]});
      RUN(launch_gemv(g, st, pdl));
    }
    if (tp && !tpf) RUN(ar_resid(Ld.down.b, trace_ptr(Ld.li[6]), fz ? m->amax_h : nullptr));
  }
  const bool fzh = m->fuse_in == 2 && !m->fr_on && !cm;
  if (tpf)
    RUN(launch_tpx_norm(m->tpx, TPX_SUM_D, m->L[c.NL - 1].down.b, m->x, c.D, m->gf, R, c.D, m->xq, m->KMAX, m->xs, st,
                        pdl));
  else if (!fzh && !fzs && !ftail)
    RUN(launch_norm_q(m->x, c.D, m->gf, R, c.D, m->xq, m->KMAX, m->xs, st, pdl, nullptr,
                      cm ? m->cap + (size_t)c.NL * c.D : nullptr, m->cap_row));
  {
    GemvArgs g;
    g.L = m->head; g.R = R; g.err = m->err; g.ldr = (int)m->trace_row;
    g.xq = m->xq; g.xs = m->xs; g.ldx = m->KMAX;
    if (fzh) { g.xin = XIN_NORM; g.x64 = m->x; g.ldx64 = c.D; g.gain = m->gf; }
    if (fzs) { g.xin = XIN_NORMST; g.x64 = m->x; g.ldx64 = c.D; g.gain = m->gf; g.nstat_in = m->nstat_a; }
    g.epi = EPI_HEAD; g.out = (want_logits || smp) ? m->logits : nullptr; g.ldo = tp ? m->vmax : c.V;
    g.raw = trace_ptr(m->n_lin - 1);
    g.head_part = m->head_part; g.head_ticket = m->head_ticket; g.next_tok = m->next_tok; g.grid = m->head_grid;
    if (tp) g.head_val = m->tp_hval;
    set_fr(g, {m->n_lin - 1});
    RUN(launch_gemv(g, st, pdl));
  }
  if (tp) {
    // greedy over the vocabulary slices: the largest value, then the lowest index holding it
    RUN(ar(m->tp_hval, m->tp_hmax, R, ncclInt64, ncclMax, 3));
    RUN(launch_tp_pick(m->tp_hval, m->tp_hmax, m->next_tok, m->v0, R, st));
    RUN(ar(m->next_tok, m->next_tok, R, ncclInt32, ncclMin, 2));
  }
  if (smp)   // replaces the head's greedy choice; advances each row's sampling position
    RUN(launch_sample(R, m->logits, c.V, c.V, m->samp_seed, m->samp_pos, true, m->samp_tnum, m->exp_t, m->next_tok,
                      st, pdl));
  if (m->fr_on) RUN(launch_fr_check(m->fr_acc, m->n_lin * RMAX, m->fr_fail, m->err, st, false));
  // note: fr_acc rows beyond R stay zero and compare equal
  if (cm)
    RUN(launch_commit_log(R, seq, pos, m->commit_seq, m->trace, m->trace_row, m->cap, m->cap_row, m->commit_log,
                          m->commit_cap, m->commit_npos, m->err, st));
#undef RUN
  return cudaSuccess;
}

__global__ void k_advance(int B, int32_t* ids, int32_t* pos, const int32_t* next, int32_t* step, int32_t* tokens,
                          int cap) {
  tl_start();
  const int r = threadIdx.x;
  const int s = *step;
  __syncthreads();
  if (r < B) {
    ids[r] = next[r];
    pos[r] += 1;
    if (s < cap) tokens[(size_t)s * B + r] = next[r];
  }
  __syncthreads();
  if (r == 0) *step = s + 1;
  tl_exit();
}

// --- graph cache: key = (R, row-array base, logits, advance, trace, freivalds)
static int run_step(exb_model* m, int R, const int32_t* ids, const int32_t* seq, const int32_t* pos, bool want_logits,
                    int advanceB) {
  if (m->c.n_experts && g_hist_row0 >= 0) {
    // direct launches: the MoE history row of this chunk is not a graph constant
    cudaError_t e = enqueue_step(m, R, ids, seq, pos, want_logits, m->st);
    if (e == cudaSuccess && advanceB > 0) {
      k_advance<<<1, 32, 0, m->st>>>(advanceB, const_cast<int32_t*>(ids), const_cast<int32_t*>(pos), m->next_tok,
                                     m->gen_step, m->gen_tokens, m->gen_cap);
      e = cudaGetLastError();
    }
    if (e != cudaSuccess) FAIL(EXB_ECUDA, std::string("step: ") + cudaGetErrorString(e));
    return EXB_OK;
  }
  const uint64_t key = ((uint64_t)R) | ((uint64_t)(want_logits ? 1 : 0) << 8) | ((uint64_t)(advanceB) << 9) |
                       ((uint64_t)(m->trace_on ? 1 : 0) << 20) | ((uint64_t)(m->fr_on ? 1 : 0) << 21) |
                       ((uint64_t)(m->commit_on ? 1 : 0) << 22) | ((uint64_t)(m->samp_active ? 1 : 0) << 23) |
                       ((uint64_t)((const char*)ids - (const char*)m->rarena) << 24);
  auto it = m->graphs.find(key);
  if (it == m->graphs.end()) {
    cudaGraph_t graph;
    CK(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = enqueue_step(m, R, ids, seq, pos, want_logits, m->st);
    if (e == cudaSuccess && advanceB > 0) {
      k_advance<<<1, 32, 0, m->st>>>(advanceB, const_cast<int32_t*>(ids), const_cast<int32_t*>(pos), m->next_tok,
                                     m->gen_step, m->gen_tokens, m->gen_cap);
      e = cudaGetLastError();
    }
    cudaError_t e2 = cudaStreamEndCapture(m->st, &graph);
    if (e != cudaSuccess) FAIL(EXB_ECUDA, std::string("step capture: ") + cudaGetErrorString(e));
    if (e2 != cudaSuccess) FAIL(EXB_ECUDA, std::string("end capture: ") + cudaGetErrorString(e2));
    {   // kernel launches of this step graph (reported by exb_step_launches)
      size_t nn = 0;
      int kernels = 0;
      if (cudaGraphGetNodes(graph, nullptr, &nn) == cudaSuccess && nn) {
        std::vector<cudaGraphNode_t> nodes(nn);
        if (cudaGraphGetNodes(graph, nodes.data(), &nn) == cudaSuccess)
          for (auto nd : nodes) {
            cudaGraphNodeType ty;
            if (cudaGraphNodeGetType(nd, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++kernels;
          }
      }
      m->step_kernels = kernels;
    }
    cudaGraphExec_t ge;
    e = cudaGraphInstantiate(&ge, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) FAIL(EXB_ECUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
    it = m->graphs.emplace(key, ge).first;
  }
  CK(cudaGraphLaunch(it->second, m->st));
  return EXB_OK;
}

static int check_device_errors(exb_model* m) {
  int bits = 0;
  CK(cudaMemcpyAsync(&bits, m->err, sizeof(int), cudaMemcpyDeviceToHost, m->st));
  CK(cudaStreamSynchronize(m->st));
  if (bits & ~ERR_FREIVALDS) {
    char buf[128];
    snprintf(buf, sizeof buf, "device error bits 0x%x (1: |V|>=2^31, 2: wait timeout, 8: bounds)", bits);
    FAIL(EXB_EDEVICE, buf);
  }
  return EXB_OK;
}

// ------------------------------------------------------------------------------------------ C ABI
#ifdef EXB_TIMELINE
namespace exb {
std::vector<int (*)(void*)>& tl_installers() {
  static std::vector<int (*)(void*)> v;
  return v;
}
int tl_register(int (*install)(void*)) {
  tl_installers().push_back(install);
  return 0;
}
}  // namespace exb
#endif

extern "C" {

const char* exb_last_error(void) { return g_err.c_str(); }
int exb_version(void) { return 1; }

int exb_gen_tensor(int kind, uint64_t seed, uint64_t stream_id, int64_t n, int64_t K, void* out, void* stream) {
  CK(gen_tensor(kind, seed, stream_id, n, K, out, (cudaStream_t)stream));
  return EXB_OK;
}

int exb_gemv(const int16_t* x16, const int8_t* wT, const int64_t* Mg, int K, int N, int64_t* out, void* stream) {
  if (!x16 || !wT || !Mg || !out || K <= 0 || N <= 0 || K % 128) FAIL(EXB_EINVAL, "exb_gemv: bad arguments (K % 128 == 0 required)");
  if (((uintptr_t)x16 | (uintptr_t)wT) & 15) FAIL(EXB_EINVAL, "exb_gemv: x16 and wT must be 16-byte aligned");
  CK(launch_gemv_op(x16, wT, Mg, K, N, out, (cudaStream_t)stream));
  return EXB_OK;
}

static size_t xq_bytes(int R, int K) { return ((size_t)R * K * sizeof(int16_t) + 255) / 256 * 256; }
static size_t xs_bytes(int R) { return ((size_t)R * sizeof(int32_t) + 255) / 256 * 256; }

static size_t scale_bytes(int K, int N) { return ((size_t)N * (size_t)(((K / 128) + 3) & ~3) * 4 + 255) / 256 * 256; }

size_t exb_linear_g128_scratch_bytes(int R, int K, int N) {
  size_t b = xq_bytes(R, K) + xs_bytes(R) + scale_bytes(K, N);
  if (R >= TC_MIN_ROWS) b += gemm_tc_digit_bytes(R, K);       // int8 digit planes for the tensor cores
  return b;
}

static int linear_common(const int64_t* x, int R, int K, const LinW& L, int64_t* y, int64_t* raw, void* scratch,
                         cudaStream_t st, bool channel) {
  int16_t* xq = (int16_t*)scratch;
  int32_t* xs = (int32_t*)((char*)scratch + xq_bytes(R, K));
  CK(launch_quant(x, K, R, K, xq, K, xs, st, false));
  if (!channel && R >= TC_MIN_ROWS && gemm_tc_supported(L, EPI_STORE)) {
    // tcgen05 path: digit planes behind the (re-pitched) scales in the scratch buffer
    void* digits = (char*)scratch + xq_bytes(R, K) + xs_bytes(R) + scale_bytes(K, L.N);
    CK(launch_digits(xq, K, R, K, digits, st));
    CK(launch_gemm_tc(digits, R, L, xs, EPI_STORE, y, L.N, raw, nullptr, L.N, nullptr, nullptr, st));
    return EXB_OK;
  }
  for (int r0 = 0; r0 < R; r0 += RMAX) {
    const int rr = R - r0 < RMAX ? R - r0 : RMAX;
    GemvArgs g;
    g.xq = xq + (size_t)r0 * K; g.xs = xs + r0; g.ldx = K; g.L = L; g.R = rr;
    g.epi = channel ? EPI_RAW : EPI_STORE;
    g.out = channel ? nullptr : y + (size_t)r0 * L.N; g.ldo = L.N;
    g.raw = raw ? raw + (size_t)r0 * L.N : nullptr; g.ldr = L.N;
    CK(launch_gemv(g, st, false));
  }
  if (channel) CK(launch_requant_channel(raw, L.N, R, L, y, L.N, xs, EPI_STORE, st, false));
  return EXB_OK;
}

int exb_linear_g128(const int64_t* x, int R, int K, const int8_t* w_NK, const int32_t* M_NG, const int64_t* bias,
                    int N, int64_t* y, int64_t* tot_out, void* scratch, void* stream) {
  if (!x || !w_NK || !M_NG || !y || !scratch || R <= 0 || K <= 0 || N <= 0 || K % 128)
    FAIL(EXB_EINVAL, "exb_linear_g128: bad arguments (K % 128 == 0 required)");
  if (((uintptr_t)w_NK | (uintptr_t)scratch) & 15) FAIL(EXB_EINVAL, "exb_linear_g128: w and scratch must be 16-byte aligned");
  LinW L; L.w = w_NK; L.Mg = M_NG; L.b = bias; L.N = N; L.K = K;
  const int G = K / 128;
  L.ldm = G;
  if ((G % 4) || ((uintptr_t)M_NG & 15)) {
    // keep the engine's layout (scale rows padded to a multiple of 4 int32, 16-byte aligned)
    int32_t* Mp = (int32_t*)((char*)scratch + xq_bytes(R, K) + xs_bytes(R));
    L.ldm = (G + 3) & ~3;
    CK(cudaMemcpy2DAsync(Mp, (size_t)L.ldm * 4, M_NG, (size_t)G * 4, (size_t)G * 4, N, cudaMemcpyDeviceToDevice,
                         (cudaStream_t)stream));
    L.Mg = Mp;
  }
  return linear_common(x, R, K, L, y, tot_out, scratch, (cudaStream_t)stream, false);
}

int exb_linear_channel(const int64_t* x, int R, int K, const int8_t* w_NK, const int64_t* M, const int64_t* bias,
                       int N, int64_t* y, int64_t* acc_out, void* scratch, void* stream) {
  if (!x || !w_NK || !M || !y || !acc_out || !scratch || R <= 0 || K <= 0 || N <= 0 || K % 16)
    FAIL(EXB_EINVAL, "exb_linear_channel: bad arguments (K % 16 == 0 and acc_out required)");
  if (((uintptr_t)w_NK | (uintptr_t)scratch) & 15) FAIL(EXB_EINVAL, "exb_linear_channel: w and scratch must be 16-byte aligned");
  std::vector<int64_t> hM(N);
  LinW L; L.w = w_NK; L.Mc = M; L.b = bias; L.N = N; L.K = K;
  // Mbits = bitlen(max M) over the layer (exact_llm.py:87)
  CK(cudaMemcpy(hM.data(), M, sizeof(int64_t) * N, cudaMemcpyDeviceToHost));
  int64_t mx = 0;
  for (int64_t v : hM) mx = v > mx ? v : mx;
  L.mbits = bitlen_host((uint64_t)mx);
  return linear_common(x, R, K, L, y, acc_out, scratch, (cudaStream_t)stream, true);
}

// Tensor-parallel shard of rank `rank` of `size` (the reference layer's natural partition):
// q heads split inside each KV group when size is a multiple of KV (7B TP8: 4/3 heads per rank
// pair, one KV head each), whole KV groups per rank when KV is a multiple of size; I split by
// 128-groups (first ranks one more); vocabulary in equal slices (the last one shorter).
// out = {qh0, qh1, kh0, kh1, ig0, ig1, v0, v1, vmax}.
static bool tp_plan(const exb_config& c, int rank, int size, int* o, std::string& why) {
  if (size < 1 || rank < 0 || rank >= size) { why = "tensor parallel: 0 <= rank < size"; return false; }
  if (size == 1) {
    const int vals[9] = {0, c.H, 0, c.KV, 0, (c.I + 127) / 128, 0, c.V, c.V};
    for (int i = 0; i < 9; ++i) o[i] = vals[i];
    return true;
  }
  if (c.lin_kind != 0 || c.n_experts) { why = "tensor parallel covers the dense group-128 models"; return false; }
  if (c.KV <= 0 || c.H % c.KV) { why = "H must be a multiple of KV"; return false; }
  const int rep = c.H / c.KV;
  int qh0, qh1, kh0, kh1;
  if (size % c.KV == 0) {
    const int mm = size / c.KV, g = rank / mm, j = rank % mm;
    if (mm > rep) { why = "more ranks per KV group than query heads"; return false; }
    const int base = rep / mm, extra = rep % mm;
    qh0 = g * rep + j * base + std::min(j, extra);
    qh1 = qh0 + base + (j < extra ? 1 : 0);
    kh0 = g; kh1 = g + 1;
  } else if (c.KV % size == 0) {
    const int per = c.KV / size;
    kh0 = rank * per; kh1 = kh0 + per;
    qh0 = kh0 * rep; qh1 = kh1 * rep;
  } else {
    why = "tensor parallel size must divide KV or be a multiple of it";
    return false;
  }
  if (((qh1 - qh0) * c.hd) % 128) { why = "query heads per rank x head_dim must be a multiple of 128"; return false; }
  if (c.I % 128 || c.I / 128 < size) { why = "I must hold at least one 128-group per rank"; return false; }
  const int G = c.I / 128, gb = G / size, ge = G % size;
  const int ig0 = rank * gb + std::min(rank, ge), ig1 = ig0 + gb + (rank < ge ? 1 : 0);
  const int vmax = (c.V + size - 1) / size, v0 = rank * vmax, v1 = std::min(c.V, v0 + vmax);
  if (v1 <= v0) { why = "vocabulary smaller than the rank count"; return false; }
  const int vals[9] = {qh0, qh1, kh0, kh1, ig0, ig1, v0, v1, vmax};
  for (int i = 0; i < 9; ++i) o[i] = vals[i];
  return true;
}

static int create_impl(const exb_config* cfg, int rank, int size, const uint8_t* uid, exb_model** out);

int exb_model_create(const exb_config* cfg, exb_model** out) { return create_impl(cfg, 0, 1, nullptr, out); }

int exb_model_create_tp(const exb_config* cfg, int rank, int size, const uint8_t* unique_id, exb_model** out) {
  if (size > 1 && !unique_id) FAIL(EXB_EINVAL, "exb_model_create_tp: unique id required");
  return create_impl(cfg, rank, size, unique_id, out);
}

int exb_tp_plan(const exb_config* cfg, int rank, int size, int32_t* out9) {
  if (!cfg || !out9) FAIL(EXB_EINVAL, "null argument");
  std::string why;
  int o[9];
  if (!tp_plan(*cfg, rank, size, o, why)) FAIL(EXB_EINVAL, why);
  for (int i = 0; i < 9; ++i) out9[i] = o[i];
  return EXB_OK;
}

int exb_tp_unique_id(uint8_t* out128) {
  if (!out128) FAIL(EXB_EINVAL, "null argument");
  if (!nccl()) FAIL(EXB_ECUDA, "libnccl.so.2 not found (tensor parallelism needs NCCL)");
  ncclUniqueId id;
  if (nccl()->get_unique_id(&id) != ncclSuccess) FAIL(EXB_ECUDA, "ncclGetUniqueId failed");
  static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
  memcpy(out128, &id, 128);
  return EXB_OK;
}

// The one-shot all-reduce's buffers: one per rank, zeroed, exported with CUDA IPC, the handles
// all-gathered with NCCL and every peer's buffer mapped here.  Collective (every rank calls it
// from create).  Any failure leaves tpc_on false: the step graph then uses NCCL.
static void tp_comm_setup(exb_model* m) {
  const int P = m->tp;
  if (P > TPC_MAX_RANKS) return;
  const int nblk = (RMAX * m->c.D + TPC_CH - 1) / TPC_CH;      // the largest call: R x D partial sums
  static_assert(RMAX <= TPX_ROWS, "exchange slots hold every row of a decode pass");
  const size_t ar_bytes = tp_comm_bytes(P, nblk);
  const size_t bytes = ar_bytes + tpx_bytes(P, m->c.D);
  bool ok = cudaMalloc(&m->tpc_local, bytes) == cudaSuccess &&
            cudaMalloc(&m->tpc_epoch, sizeof(unsigned long long) * nblk) == cudaSuccess &&
            cudaMalloc(&m->tpx_ep, sizeof(unsigned long long) * 4) == cudaSuccess &&
            cudaMalloc(&m->tpx_tickets, sizeof(unsigned int) * 2) == cudaSuccess &&
            cudaMalloc(&m->tpx_dev, sizeof(TpX)) == cudaSuccess &&
            cudaMemset(m->tpc_local, 0, bytes) == cudaSuccess &&
            cudaMemset(m->tpc_epoch, 0, sizeof(unsigned long long) * nblk) == cudaSuccess &&
            cudaMemset(m->tpx_ep, 0, sizeof(unsigned long long) * 4) == cudaSuccess &&
            cudaMemset(m->tpx_tickets, 0, sizeof(unsigned int) * 2) == cudaSuccess;
  cudaIpcMemHandle_t mine;
  if (ok) ok = cudaIpcGetMemHandle(&mine, m->tpc_local) == cudaSuccess;
  // every rank takes part in the exchange, also after a local failure (a zeroed handle marks it)
  if (!ok) memset(&mine, 0, sizeof mine);
  std::vector<cudaIpcMemHandle_t> all(P);
  char* dbuf = nullptr;
  if (cudaMalloc(&dbuf, sizeof(cudaIpcMemHandle_t) * (P + 1)) != cudaSuccess) { cudaGetLastError(); return; }
  cudaMemcpy(dbuf + sizeof(cudaIpcMemHandle_t) * P, &mine, sizeof mine, cudaMemcpyHostToDevice);
  const bool gathered = nccl()->all_gather(dbuf + sizeof(cudaIpcMemHandle_t) * P, dbuf, sizeof(cudaIpcMemHandle_t),
                                           ncclUint8, m->comm, m->st) == ncclSuccess;
  if (gathered) cudaMemcpyAsync(all.data(), dbuf, sizeof(cudaIpcMemHandle_t) * P, cudaMemcpyDeviceToHost, m->st);
  cudaStreamSynchronize(m->st);
  cudaFree(dbuf);
  ok = ok && gathered;
  const cudaIpcMemHandle_t zero{};
  for (int q = 0; q < P && ok; ++q) {
    if (memcmp(&all[q], &zero, sizeof zero) == 0) ok = false;
    if (q != m->tp_rank && ok) {       // mapping a peer's buffer enables the peer access it needs
      void* p = nullptr;
      ok = cudaIpcOpenMemHandle(&p, all[q], cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
      m->tpc.base[q] = (char*)p;
    }
  }
  // agree: the kernel runs only if every rank mapped every peer (an int MIN over the ranks)
  int* flag = nullptr;
  int v = ok ? 1 : 0;
  if (cudaMalloc(&flag, sizeof(int)) == cudaSuccess) {
    cudaMemcpy(flag, &v, sizeof v, cudaMemcpyHostToDevice);
    if (nccl()->all_reduce(flag, flag, 1, ncclInt32, ncclMin, m->comm, m->st) == ncclSuccess) {
      cudaMemcpyAsync(&v, flag, sizeof v, cudaMemcpyDeviceToHost, m->st);
      cudaStreamSynchronize(m->st);
    } else {
      v = 0;
    }
    cudaFree(flag);
  } else {
    v = 0;
  }
  cudaGetLastError();
  m->tpc.rank = m->tp_rank; m->tpc.size = P; m->tpc.nblk = nblk;
  m->tpc.base[m->tp_rank] = m->tpc_local;
  m->tpc.epoch = m->tpc_epoch; m->tpc.err = m->err;
  m->tpc_on = v == 1;
  m->tpx.rank = m->tp_rank; m->tpx.size = P; m->tpx.D = m->c.D;
  for (int q = 0; q < P; ++q) m->tpx.base[q] = m->tpc.base[q] ? m->tpc.base[q] + ar_bytes : nullptr;
  m->tpx.ep = m->tpx_ep; m->tpx.err = m->err;
  if (m->tpc_on) m->tpc_on = cudaMemcpy(m->tpx_dev, &m->tpx, sizeof(TpX), cudaMemcpyHostToDevice) == cudaSuccess;
}

static int create_impl(const exb_config* cfg, int rank, int size, const uint8_t* uid, exb_model** out) {
  if (!cfg || !out) FAIL(EXB_EINVAL, "null argument");
  int plan[9];
  {
    std::string why;
    if (!tp_plan(*cfg, rank, size, plan, why)) FAIL(EXB_EINVAL, why);
  }
  // this rank's architecture: its heads, MLP groups and vocabulary slice
  exb_config cl = *cfg;
  if (size > 1) {
    cl.H = plan[1] - plan[0]; cl.KV = plan[3] - plan[2]; cl.I = (plan[5] - plan[4]) * 128; cl.V = plan[7] - plan[6];
  }
  const exb_config& c = cl;
  if (c.D <= 0 || c.H <= 0 || c.KV <= 0 || c.hd <= 0 || c.I <= 0 || c.V <= 0 || c.NL <= 0) FAIL(EXB_EINVAL, "bad dims");
  if (c.H % c.KV || c.H / c.KV > 8) FAIL(EXB_EINVAL, "H must be a multiple of KV with at most 8 query heads per KV head");
  if (c.hd % 16 || c.hd > 128) FAIL(EXB_EINVAL, "head_dim must be a multiple of 16 and <= 128");
  if (c.n_experts && (c.lin_kind == 0 || c.n_experts > MOE_MAX_EXPERTS || c.topk < 1 || c.topk > MOE_MAX_TOPK ||
                      c.topk > c.n_experts || c.moe_I <= 0 || c.shared_I <= 0 || c.moe_I % 16 || c.shared_I % 16))
    FAIL(EXB_EINVAL, "MoE: per-channel linears, 1 <= topk <= min(8, n_experts), n_experts <= 128, "
                     "expert and shared widths multiples of 16");
  if (c.max_batch <= 0 || c.max_seq <= 0 || c.rope_len < c.max_seq) FAIL(EXB_EINVAL, "bad capacities");
  const int gk = c.lin_kind == 0 ? 128 : 16;
  if (c.D % gk || (c.H * c.hd) % gk || c.I % gk) FAIL(EXB_EINVAL, "D, H*hd and I must be multiples of 128 (group) or 16 (channel)");
  exb_model* m = new exb_model();
  m->c = c;
  m->cg = *cfg;
  m->tp = size; m->tp_rank = rank;
  m->qh0 = plan[0]; m->qh1 = plan[1]; m->kh0 = plan[2]; m->kh1 = plan[3];
  m->ig0 = plan[4]; m->ig1 = plan[5]; m->v0 = plan[6]; m->v1 = plan[7]; m->vmax = plan[8];
  m->group = c.lin_kind == 0;
  m->Nqkv = (c.H + 2 * c.KV) * c.hd;
  m->KMAX = std::max(std::max(c.D, c.H * c.hd), c.I);
  m->NMAX = std::max(std::max(m->Nqkv, 2 * c.I), c.V);
  if (c.n_experts) m->NMAX = std::max(m->NMAX, 2 * std::max(c.moe_I, c.shared_I));
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  m->head_grid = std::min(2 * sms, (c.V + 3) / 4);   // the GEMV runs two CTAs per SM
  m->sms = sms;
  plan_weights(m);
  m->wbytes = m->woff;
  plan_lins(m);
  plan_runtime(m);
  m->rbytes = m->roff + (size_t)m->n_lin * ((2 * (size_t)m->NMAX + 2 * (size_t)m->KMAX) * 4 + 512) + 4096;
  cudaError_t e = cudaMalloc(&m->warena, m->wbytes);
  if (e == cudaSuccess) e = cudaMalloc(&m->rarena, m->rbytes);
  if (e != cudaSuccess) {
    cudaFree(m->warena);
    delete m;
    FAIL(EXB_ENOMEM, std::string("device allocation failed: ") + cudaGetErrorString(e));
  }
  plan_weights(m);
  plan_lins(m);
  plan_runtime(m);
  cudaMemset(m->rarena, 0, m->rbytes);
  cudaMemset(m->warena, 0, m->wbytes);
  cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking);
  cudaMallocHost(&m->h_ids, sizeof(int32_t) * RMAX * 3);
  m->h_seq = m->h_ids + RMAX; m->h_pos = m->h_ids + 2 * RMAX;
  m->seq_len.assign(c.max_batch, 0);
  if (size > 1) {
    ncclUniqueId id;
    memcpy(&id, uid, sizeof id);
    // collective: every rank of the group calls this concurrently
    if (!nccl() || nccl()->comm_init_rank(&m->comm, size, id, rank) != ncclSuccess) {
      exb_model_destroy(m);
      FAIL(EXB_ECUDA, "ncclCommInitRank failed");
    }
    tp_comm_setup(m);            // collective; NCCL stays the all-reduce when the peers cannot be mapped
  }
  *out = m;
  return EXB_OK;
}

void exb_model_destroy(exb_model* m) {
  if (!m) return;
  for (int q = 0; q < TPC_MAX_RANKS; ++q)
    if (q != m->tp_rank && m->tpc.base[q]) cudaIpcCloseMemHandle(m->tpc.base[q]);
  cudaFree(m->tpc_local);
  cudaFree(m->tpc_epoch);
  cudaFree(m->tpx_ep);
  cudaFree(m->tpx_tickets);
  cudaFree(m->tpx_dev);
  for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
  if (m->st) cudaStreamSynchronize(m->st);
  cudaFree(m->warena);
  cudaFree(m->rarena);
  cudaFree(m->commit_log);
  cudaFree(m->commit_lin);
  cudaFree(m->ver_emb_r);
  cudaFree(m->ver_emb_de);
  cudaFree(m->gen_tokens);
  cudaFree(m->emb_q16);
  if (m->comm && nccl()) nccl()->comm_destroy(m->comm);
  cudaFree(m->p_arena);
  if (m->p_hrows) cudaFreeHost(m->p_hrows);
  if (m->h_ids) cudaFreeHost(m->h_ids);
  if (m->st) cudaStreamDestroy(m->st);
  delete m;
}

static int to_i32_device(exb_model* m, const int64_t* h, size_t n, int32_t* d) {
  std::vector<int32_t> t(n);
  for (size_t i = 0; i < n; ++i) {
    if (h[i] > INT32_MAX || h[i] < INT32_MIN) FAIL(EXB_EINVAL, "table value does not fit int32");
    t[i] = (int32_t)h[i];
  }
  CK(cudaMemcpyAsync(d, t.data(), n * 4, cudaMemcpyHostToDevice, m->st));
  CK(cudaStreamSynchronize(m->st));
  return EXB_OK;
}

int exb_model_set_tables(exb_model* m, const int64_t* exp_t, const int64_t* silu_t, const int64_t* sig_t,
                         const int64_t* cos_t, const int64_t* sin_t) {
  if (!m || !exp_t || !silu_t || !cos_t || !sin_t) FAIL(EXB_EINVAL, "null table");
  int rc;
  if ((rc = to_i32_device(m, exp_t, EXP_LEN_H, m->exp_t))) return rc;
  if ((rc = to_i32_device(m, silu_t, SILU_LEN_H, m->silu_t))) return rc;
  if (sig_t && (rc = to_i32_device(m, sig_t, SILU_LEN_H, m->sig_t))) return rc;
  const size_t n = (size_t)m->c.rope_len * (m->c.hd / 2);
  if ((rc = to_i32_device(m, cos_t, n, m->cos_t))) return rc;
  if ((rc = to_i32_device(m, sin_t, n, m->sin_t))) return rc;
  return EXB_OK;
}

// copy a logical (N x row_bytes) host tensor into fused rows row0 + i*step of a device matrix whose
// rows are dst_row_bytes apart
static int put_rows(exb_model* m, void* dst_base, size_t dst_row_bytes, int row0, int step, const void* src, int N,
                    size_t row_bytes = 0, cudaMemcpyKind kind = cudaMemcpyHostToDevice) {
  if (!row_bytes) row_bytes = dst_row_bytes;
  char* dst = (char*)dst_base + (size_t)row0 * dst_row_bytes;
  CK(cudaMemcpy2DAsync(dst, dst_row_bytes * step, src, row_bytes, row_bytes, N, kind, m->st));
  return EXB_OK;
}

static LinInfo* find_lin(exb_model* m, const std::string& nm) {
  for (auto& l : m->lins)
    if (l.name == nm) return &l;
  return nullptr;
}

// Tensor parallel: cut this rank's window out of a global (rows x cols) row-major host tensor of
// `esz`-byte elements (rows [r0, r0 + nr), columns [c0, c0 + nc)).
static std::vector<char> host_window(const void* src, size_t cols, size_t esz, size_t r0, size_t nr, size_t c0, size_t nc) {
  std::vector<char> out(nr * nc * esz);
  for (size_t r = 0; r < nr; ++r)
    memcpy(out.data() + r * nc * esz, (const char*)src + ((r0 + r) * cols + c0) * esz, nc * esz);
  return out;
}

static int set_tensor_local(exb_model* m, const std::string& name, const void* host, size_t bytes);

int exb_model_set_tensor(exb_model* m, const char* name_c, const void* host, size_t bytes) {
  if (!m || !name_c || !host) FAIL(EXB_EINVAL, "null argument");
  const std::string name(name_c);
  if (m->tp == 1) return set_tensor_local(m, name, host, bytes);
  // global tensors in, this rank's slices stored
  const exb_config& g = m->cg;
  if (name == "head.w") {
    if (bytes != (size_t)g.V * g.D) FAIL(EXB_EINVAL, "head.w: wrong size");
    auto w = host_window(host, g.D, 1, m->v0, m->v1 - m->v0, 0, g.D);
    return set_tensor_local(m, name, w.data(), w.size());
  }
  if (name == "head.M") {
    if (bytes != (size_t)g.V * 8) FAIL(EXB_EINVAL, "head.M: wrong size");
    auto w = host_window(host, 1, 8, m->v0, m->v1 - m->v0, 0, 1);
    return set_tensor_local(m, name, w.data(), w.size());
  }
  const size_t d1 = name.find('.'), d2 = name.find('.', d1 + 1);
  if (name[0] == 'L' && d2 != std::string::npos) {
    LinInfo* L = find_lin(m, name.substr(0, d2));
    if (L && (L->Ng != L->N || L->Kg != L->K)) {
      const std::string part = name.substr(d2 + 1);
      if (part == "w") {
        if (bytes != (size_t)L->Ng * L->Kg) FAIL(EXB_EINVAL, name + ": wrong size (global shape)");
        auto w = host_window(host, L->Kg, 1, L->r_lo, L->N, L->c_lo, L->K);
        return set_tensor_local(m, name, w.data(), w.size());
      }
      if (part == "M") {
        const int Gg = L->Kg / 128;
        if (bytes != (size_t)L->Ng * Gg * 4) FAIL(EXB_EINVAL, name + ": wrong size (global shape, int32 N x K/128)");
        auto w = host_window(host, Gg, 4, L->r_lo, L->N, L->c_lo / 128, L->K / 128);
        return set_tensor_local(m, name, w.data(), w.size());
      }
      if (part == "b") {
        if (bytes != (size_t)L->Ng * 8) FAIL(EXB_EINVAL, name + ": wrong size (global shape)");
        auto w = host_window(host, 1, 8, L->r_lo, L->N, 0, 1);
        return set_tensor_local(m, name, w.data(), w.size());
      }
    }
  }
  return set_tensor_local(m, name, host, bytes);
}

static int set_tensor_local(exb_model* m, const std::string& name, const void* host, size_t bytes) {
  const exb_config& c = m->c;
  auto need = [&](size_t n) -> bool { return bytes == n; };
  if (name == "emb_q16") {
    if (!need((size_t)m->cg.V * c.D * 8)) FAIL(EXB_EINVAL, "emb_q16: wrong size");
    if (!m->emb_q16) CK(cudaMalloc(&m->emb_q16, bytes));
    CK(cudaMemcpyAsync(m->emb_q16, host, bytes, cudaMemcpyHostToDevice, m->st));
  } else if (name == "emb") {
    if (!need((size_t)m->cg.V * c.D)) FAIL(EXB_EINVAL, "emb: wrong size");
    CK(cudaMemcpyAsync(m->emb, host, bytes, cudaMemcpyHostToDevice, m->st));
  } else if (name == "gf") {
    if (!need((size_t)c.D * 8)) FAIL(EXB_EINVAL, "gf: wrong size");
    CK(cudaMemcpyAsync(m->gf, host, bytes, cudaMemcpyHostToDevice, m->st));
  } else if (name == "head.w") {
    if (c.tie) FAIL(EXB_EINVAL, "head.w: tied model");
    if (!need((size_t)c.V * c.D)) FAIL(EXB_EINVAL, "head.w: wrong size");
    CK(cudaMemcpyAsync((void*)m->head.w, host, bytes, cudaMemcpyHostToDevice, m->st));
  } else if (name == "head.M") {
    if (!need((size_t)c.V * 8)) FAIL(EXB_EINVAL, "head.M: wrong size");
    CK(cudaMemcpyAsync((void*)m->head.Mc, host, bytes, cudaMemcpyHostToDevice, m->st));
  } else {
    // L{i}.xxx
    if (name.size() < 3 || name[0] != 'L') FAIL(EXB_EINVAL, "unknown tensor " + name);
    const size_t dot = name.find('.');
    const int li = atoi(name.substr(1, dot - 1).c_str());
    if (li < 0 || li >= c.NL || dot == std::string::npos) FAIL(EXB_EINVAL, "bad layer in " + name);
    LayerDev& Ld = m->L[li];
    const std::string rest = name.substr(dot + 1);
    if (rest == "g1" || rest == "g2") {
      if (!need((size_t)c.D * 8)) FAIL(EXB_EINVAL, name + ": wrong size");
      CK(cudaMemcpyAsync(rest == "g1" ? Ld.g1 : Ld.g2, host, bytes, cudaMemcpyHostToDevice, m->st));
    } else {
      const size_t d2 = rest.find('.');
      if (d2 == std::string::npos) FAIL(EXB_EINVAL, "unknown tensor " + name);
      LinInfo* L = find_lin(m, name.substr(0, dot + 1 + d2));
      if (!L) FAIL(EXB_EINVAL, "unknown linear in " + name);
      const std::string part = rest.substr(d2 + 1);
      LinW& F = *L->fused;
      if (part == "w") {
        if (!need((size_t)L->N * L->K)) FAIL(EXB_EINVAL, name + ": wrong size");
        return put_rows(m, (void*)F.w, (size_t)L->K, L->row0, L->row_step, host, L->N);
      } else if (part == "M") {
        if (m->group) {
          if (!need((size_t)L->N * (L->K / 128) * 4)) FAIL(EXB_EINVAL, name + ": wrong size (int32 N x K/128)");
          return put_rows(m, (void*)F.Mg, (size_t)F.ldm * 4, L->row0, L->row_step, host, L->N, (size_t)(L->K / 128) * 4);
        }
        if (!need((size_t)L->N * 8)) FAIL(EXB_EINVAL, name + ": wrong size (int64 N)");
        return put_rows(m, (void*)F.Mc, 8, L->row0, L->row_step, host, L->N);
      } else if (part == "b") {
        if (!F.b) FAIL(EXB_EINVAL, name + ": this linear has no bias");
        if (!need((size_t)L->N * 8)) FAIL(EXB_EINVAL, name + ": wrong size");
        return put_rows(m, (void*)F.b, 8, L->row0, L->row_step, host, L->N);
      } else {
        FAIL(EXB_EINVAL, "unknown tensor " + name);
      }
    }
  }
  return EXB_OK;
}

// Stream ids of the synthetic generator (same numbering as the test oracle's generator).
static uint64_t layer_stream(int li, int off) { return (uint64_t)li * 64 + off; }

int exb_model_generate(exb_model* m, uint64_t seed) {
  if (!m) FAIL(EXB_EINVAL, "null model");
  const exb_config& c = m->c;
  size_t maxn = (size_t)m->cg.V * c.D;
  for (auto& l : m->lins) maxn = std::max(maxn, (size_t)l.Ng * l.Kg);
  void* tmp = nullptr;
  void* win = nullptr;                       // tensor parallel: this rank's window of a global tensor
  CK(cudaMallocAsync(&tmp, maxn * 8, m->st));
  if (m->tp > 1) CK(cudaMallocAsync(&win, maxn * 8, m->st));
  // global (rows x cols) device tensor of esz-byte elements -> its [r0, +nr) x [c0, +nc) window
  auto window = [&](const void* src, size_t cols, size_t esz, size_t r0, size_t nr, size_t c0, size_t nc) -> const void* {
    if (m->tp == 1) return src;
    cudaMemcpy2DAsync(win, nc * esz, (const char*)src + (r0 * cols + c0) * esz, cols * esz, nc * esz, nr,
                      cudaMemcpyDeviceToDevice, m->st);
    return win;
  };
  static const std::map<std::string, int> LS = {{"q", 2}, {"k", 5}, {"v", 8}, {"o", 11}, {"gate", 14}, {"up", 17},
                                                 {"down", 20}, {"router", 23}, {"sgate", 26}, {"sg", 29}, {"su", 32},
                                                 {"sd", 35}};
  for (auto& L : m->lins) {
    if (L.name == "head") continue;
    const int li = atoi(L.name.c_str() + 1);
    const std::string nm = L.name.substr(L.name.find('.') + 1);
    uint64_t s0;
    if (nm[0] == 'e' && nm.size() > 1 && isdigit((unsigned char)nm[1])) {
      // expert e, linear j in (g, u, d): stream (1 << 24) + layer * 4096 + e * 16 + j * 4
      const int e = atoi(nm.c_str() + 1);
      const char part = nm[nm.find('.') + 1];
      const int j = part == 'g' ? 0 : part == 'u' ? 1 : 2;
      s0 = (1ull << 24) + (uint64_t)li * 4096 + (uint64_t)e * 16 + (uint64_t)j * 4;
    } else {
      s0 = layer_stream(li, LS.at(nm));
    }
    LinW& F = *L.fused;
    CK(gen_tensor(GEN_WEIGHT, seed, s0, (int64_t)L.Ng * L.Kg, L.Kg, tmp, m->st));
    const void* src = window(tmp, L.Kg, 1, L.r_lo, L.N, L.c_lo, L.K);
    CK(cudaMemcpy2DAsync((char*)F.w + (size_t)L.row0 * L.K, (size_t)L.K * L.row_step, src, L.K, L.K, L.N,
                         cudaMemcpyDeviceToDevice, m->st));
    if (m->group) {
      const int G = L.K / 128, Gg = L.Kg / 128;
      CK(gen_tensor(GEN_SCALE32, seed, s0 + 1, (int64_t)L.Ng * Gg, L.Kg, tmp, m->st));
      src = window(tmp, Gg, 4, L.r_lo, L.N, L.c_lo / 128, G);
      int rc = put_rows(m, (void*)F.Mg, (size_t)F.ldm * 4, L.row0, L.row_step, src, L.N, (size_t)G * 4,
                        cudaMemcpyDeviceToDevice);
      if (rc) return rc;
    } else {
      CK(gen_tensor(GEN_SCALE64, seed, s0 + 1, L.Ng, L.Kg, tmp, m->st));
      src = window(tmp, 1, 8, L.r_lo, L.N, 0, 1);
      CK(cudaMemcpy2DAsync((char*)F.Mc + (size_t)L.row0 * 8, (size_t)8 * L.row_step, src, 8, 8, L.N,
                           cudaMemcpyDeviceToDevice, m->st));
    }
    if (F.b) {
      CK(gen_tensor(GEN_BIAS, seed, s0 + 2, L.Ng, 0, tmp, m->st));
      src = window(tmp, 1, 8, L.r_lo, L.N, 0, 1);
      CK(cudaMemcpy2DAsync((char*)F.b + (size_t)L.row0 * 8, (size_t)8 * L.row_step, src, 8, 8, L.N,
                           cudaMemcpyDeviceToDevice, m->st));
    }
  }
  for (int i = 0; i < c.NL; ++i) {
    CK(gen_tensor(GEN_GAIN, seed, layer_stream(i, 0), c.D, 0, m->L[i].g1, m->st));
    CK(gen_tensor(GEN_GAIN, seed, layer_stream(i, 1), c.D, 0, m->L[i].g2, m->st));
  }
  const uint64_t S_EMB = 1ull << 20;
  const int Vg = m->cg.V, Vl = m->v1 - m->v0;
  CK(gen_tensor(GEN_WEIGHT, seed, S_EMB, (int64_t)Vg * c.D, c.D, m->emb, m->st));
  CK(gen_tensor(GEN_GAIN, seed, S_EMB + 1, c.D, 0, m->gf, m->st));
  if (!c.tie) {
    CK(gen_tensor(GEN_WEIGHT, seed, S_EMB + 2, (int64_t)Vg * c.D, c.D, tmp, m->st));
    CK(cudaMemcpyAsync((void*)m->head.w, (const char*)tmp + (size_t)m->v0 * c.D, (size_t)Vl * c.D,
                       cudaMemcpyDeviceToDevice, m->st));
  }
  CK(gen_tensor(GEN_SCALE64, seed, S_EMB + 3, Vg, c.D, tmp, m->st));
  CK(cudaMemcpyAsync((void*)m->head.Mc, (const char*)tmp + (size_t)m->v0 * 8, (size_t)Vl * 8, cudaMemcpyDeviceToDevice,
                     m->st));
  if (win) CK(cudaFreeAsync(win, m->st));
  CK(cudaFreeAsync(tmp, m->st));
  CK(cudaStreamSynchronize(m->st));
  return EXB_OK;
}

int exb_model_finalize(exb_model* m) {
  if (!m) FAIL(EXB_EINVAL, "null model");
  const exb_config& c = m->c;
  CK(cudaStreamSynchronize(m->st));
  // per-channel drop rule (exact_llm.py:93): provably inactive when
  // bitlen(K * 32767 * 127) + bitlen(max M) <= 62 for every row
  for (auto& L : m->lins) {
    LinW& F = *L.fused;
    if (F.Mc) {
      // logical rows of this linear inside the fused scale vector
      std::vector<int64_t> h((size_t)F.N);
      CK(cudaMemcpy(h.data(), F.Mc, 8 * (size_t)F.N, cudaMemcpyDeviceToHost));
      int64_t mx = 0;
      for (int i = 0; i < L.N; ++i) mx = std::max(mx, h[(size_t)L.row0 + (size_t)i * L.row_step]);
      L.mbits = bitlen_host((uint64_t)mx);
      const int accbits = bitlen_host((uint64_t)L.K * 32767ull * 127ull);
      if (accbits + L.mbits > 62) F.nodrop = false;
      F.mbits = std::max(F.mbits, L.mbits);
    }
  }
  CK(cudaStreamSynchronize(m->st));
  auto moe_lin = [&](const std::string& nm) {
    const std::string t = nm.substr(nm.find('.') + 1);
    return t == "router" || t == "sgate" || t == "sg" || t == "su" || t == "sd" || (t[0] == 'e' && isdigit((unsigned char)t[1]));
  };
  if (c.n_experts) {
    // the MoE linears apply the drop rule per row on the device: record each logical linear's
    // bitlen(max M) in the expert tables
    std::map<std::string, int> mb;
    for (auto& L : m->lins) mb[L.name] = L.mbits;
    for (int i = 0; i < c.NL; ++i) {
      LayerDev& Ld = m->L[i];
      const std::string p = "L" + std::to_string(i) + ".";
      Ld.router.mbits = mb[p + "router"];
      Ld.sgate.mbits = mb[p + "sgate"];
      std::vector<ExpertW> tab(c.n_experts + 1);
      for (int e = 0; e <= c.n_experts; ++e) {
        const bool sh = e == c.n_experts;
        const std::string q = sh ? p : p + "e" + std::to_string(e) + ".";
        ExpertW& X = tab[e];
        X.w_gu = Ld.exgu[e].w; X.M_gu = Ld.exgu[e].Mc; X.w_d = Ld.exd[e].w; X.M_d = Ld.exd[e].Mc;
        X.I = sh ? c.shared_I : c.moe_I;
        X.mb_g = mb[q + (sh ? "sg" : "g")]; X.mb_u = mb[q + (sh ? "su" : "u")]; X.mb_d = mb[q + (sh ? "sd" : "d")];
      }
      CK(cudaMemcpy(Ld.ex_dev, tab.data(), sizeof(ExpertW) * tab.size(), cudaMemcpyHostToDevice));
    }
  }
  for (auto& L : m->lins)
    if (L.fused->Mc && !L.fused->nodrop && !moe_lin(L.name))
      FAIL(EXB_EINVAL, "per-channel linear " + L.name + " may trigger the overflow drop rule; the fused decode path "
                       "requires bitlen(K*32767*127) + bitlen(max M) <= 62");
  if (const char* v = getenv("EXB_FUSE")) m->fuse_in = atoi(v);
  if (const char* v = getenv("EXB_TCD")) m->tc_decode = atoi(v) != 0;
  m->finalized = true;
  return EXB_OK;
}

int exb_seq_reset(exb_model* m, int seq) {
  if (!m || seq < 0 || seq >= m->c.max_batch) FAIL(EXB_EINVAL, "bad sequence slot");
  m->seq_len[seq] = 0;
  return EXB_OK;
}
int exb_seq_len(exb_model* m, int seq) {
  if (!m || seq < 0 || seq >= m->c.max_batch) return -1;
  return m->seq_len[seq];
}

// ------------------------------------------------------------------------------------------ prefill
// Chunks of many rows (prompt tokens, batched rows) run every linear on the tcgen05 GEMM
// (gemm_tc.cu) instead of the CUDA-core GEMV: the same kernels for norm, RoPE/cache, attention
// and qrow, the same integer results.  Rows keep their order; rows of one sequence in one chunk
// see each other through the KV cache (written before the attention launch).
static constexpr int PCH = 512;            // rows per tensor-core chunk (layout of the host staging rows)

// Rows per chunk: 512 (a 512-token prompt is one chunk, and the narrow linears q|k|v, o and down
// get 4 activation tiles per weight tile instead of 2); MoE blocks take at most MOE_ROWS rows.
static int chunk_rows(const exb_model* m) { return m->c.n_experts ? std::min(PCH, MOE_ROWS) : PCH; }

static int prefill_alloc(exb_model* m) {
  if (m->pch) return EXB_OK;
  const exb_config& c = m->c;
  const int P = chunk_rows(m), Hd = c.H * c.hd;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = (off + bytes + 255) & ~size_t(255); return o; };
  const size_t o_rows = take(sizeof(int32_t) * 3 * PCH), o_x = take(8ull * P * c.D), o_qkv = take(8ull * P * m->Nqkv),
               o_ao = take(8ull * P * Hd), o_hb = take(8ull * P * c.I), o_raw = take(8ull * P * c.V),
               o_xq = take(2ull * P * m->KMAX), o_qq = take(2ull * P * Hd), o_xs = take(4ull * P),
               o_qs = take(4ull * P * c.H), o_next = take(4ull * P), o_dig = take(gemm_tc_digit_bytes(P, m->KMAX)),
               o_amax = take(8ull * P);
  CK(cudaMalloc(&m->p_arena, off));
  CK(cudaMallocHost(&m->p_hrows, sizeof(int32_t) * 3 * PCH));
  char* b = m->p_arena;
  m->p_rows = (int32_t*)(b + o_rows); m->p_x = (int64_t*)(b + o_x); m->p_qkv = (int64_t*)(b + o_qkv);
  m->p_ao = (int64_t*)(b + o_ao); m->p_hb = (int64_t*)(b + o_hb); m->p_raw = (int64_t*)(b + o_raw);
  m->p_xq = (int16_t*)(b + o_xq); m->p_qq = (int16_t*)(b + o_qq); m->p_xs = (int32_t*)(b + o_xs);
  m->p_qs = (int32_t*)(b + o_qs); m->p_next = (int32_t*)(b + o_next); m->p_dig = b + o_dig;
  m->p_amax = (unsigned long long*)(b + o_amax);
  m->pch = P;
  return EXB_OK;
}

// one chunk of R rows (R <= PCH): host ids / seq / pos already in m->p_hrows
static int prefill_chunk(exb_model* m, int R, int64_t* logits_host, int32_t* next_host) {
  const exb_config& c = m->c;
  cudaStream_t st = m->st;
  const int D = c.D, Hd = c.H * c.hd, I = c.I;
  CK(cudaMemcpyAsync(m->p_rows, m->p_hrows, sizeof(int32_t) * 3 * PCH, cudaMemcpyHostToDevice, st));
  const int32_t* ids = m->p_rows;
  const int32_t* seq = m->p_rows + PCH;
  const int32_t* pos = m->p_rows + 2 * PCH;
  if (m->emb_q16) CK(launch_embed64(m->emb_q16, ids, R, D, m->p_x, st, false));
  else CK(launch_embed(m->emb, c.emb_shift, ids, R, D, m->p_x, st, false));
  AttnArgs aa;
  aa.qkv = m->p_qkv; aa.ldqkv = m->Nqkv; aa.row_seq = seq; aa.row_pos = pos;
  aa.cos_t = m->cos_t; aa.sin_t = m->sin_t; aa.qq = m->p_qq; aa.qs = m->p_qs; aa.exp_t = m->exp_t;
  aa.out = m->p_ao; aa.ldo = Hd; aa.R = R; aa.H = c.H; aa.KV = c.KV; aa.hd = c.hd; aa.Smax = c.max_seq;
  aa.Tmax = c.rope_len; aa.err = m->err;
  aa.inv = (int64_t)std::nearbyint(65536.0 / std::sqrt((double)c.hd));
  // a chunk of consecutive positions of one sequence takes the query-tile attention kernel
  bool one_seq = m->attn_prefill;
  for (int r = 1; r < R && one_seq; ++r)
    one_seq = m->p_hrows[PCH + r] == m->p_hrows[PCH] && m->p_hrows[2 * PCH + r] == m->p_hrows[2 * PCH] + r;
  // the row kernels before the group-128 linears write the int8 digit planes themselves (planes of
  // Tpad rows; the padding rows' sums are never stored); per-channel linears take the digit kernel
  const int Tpad = (R + TC_PAD_ROWS - 1) / TC_PAD_ROWS * TC_PAD_ROWS;
  uint8_t* dig = m->group ? static_cast<uint8_t*>(m->p_dig) : nullptr;
  auto lin = [&](const int16_t* xq, int K, const LinW& L, int epi, int64_t* out, int ldo,
                 unsigned long long* amax = nullptr) -> cudaError_t {
    cudaError_t e = cudaSuccess;
    if (!dig) e = launch_digits(xq, K, R, K, m->p_dig, st);
    if (e != cudaSuccess) return e;
    if (L.Mg || epi == EPI_RAW)
      return launch_gemm_tc(m->p_dig, R, L, m->p_xs, epi, out, ldo, epi == EPI_RAW ? out : nullptr, nullptr, ldo,
                            m->silu_t, m->err, st, nullptr, amax);
    // per-channel linear: raw sums on the tensor cores, then the QLin requant (exact_llm.py:89-96)
    e = launch_gemm_tc(m->p_dig, R, L, m->p_xs, EPI_RAW, m->p_raw, L.N, m->p_raw, nullptr, L.N, nullptr, m->err, st);
    if (e != cudaSuccess) return e;
    return launch_requant_channel(m->p_raw, L.N, R, L, out, ldo, m->p_xs, epi, st, false);
  };
  for (int i = 0; i < c.NL; ++i) {
    LayerDev& Ld = m->L[i];
    const size_t kvoff = m->kv_layer_elems * i;
    aa.kc = m->kc + kvoff; aa.vc = m->vc + kvoff;
    aa.ks = m->ks + (size_t)c.max_batch * c.KV * c.max_seq * i;
    CK(launch_norm_q(m->p_x, D, Ld.g1, R, D, m->p_xq, D, m->p_xs, st, false, dig, nullptr, 0, Tpad));
    CK(lin(m->p_xq, D, Ld.qkv, EPI_STORE, m->p_qkv, m->Nqkv));
    CK(launch_rope_cache(aa, st, false));
    if (one_seq) CK(launch_attn_prefill(aa, st));       // query tiles share the cached K/V rows
    else CK(launch_attn_decode(aa, st, false));
    CK(launch_quant(m->p_ao, Hd, R, Hd, m->p_xq, Hd, m->p_xs, st, false, dig, Tpad));
    CK(lin(m->p_xq, Hd, Ld.o, EPI_RESID, m->p_x, D));
    CK(launch_norm_q(m->p_x, D, Ld.g2, R, D, m->p_xq, D, m->p_xs, st, false, c.n_experts ? nullptr : dig, nullptr, 0,
                     Tpad));
    if (c.n_experts) {
      CK(launch_moe(moe_args(m, i, R, m->p_xq, D, m->p_xs, g_hist_row0), m->p_x, D, st));
      continue;
    }
    if (dig) {
      // gate|up publishes each row's max |h|; the qrow of h then runs split over slices of the row
      CK(cudaMemsetAsync(m->p_amax, 0, sizeof(unsigned long long) * R, st));
      CK(lin(m->p_xq, D, Ld.gu, EPI_SWIGLU, m->p_hb, I, m->p_amax));
      CK(launch_quant_known(m->p_hb, I, R, I, m->p_amax, m->p_xq, I, m->p_xs, st, false, dig, Tpad));
    } else {
      CK(lin(m->p_xq, D, Ld.gu, EPI_SWIGLU, m->p_hb, I));
      CK(launch_quant(m->p_hb, I, R, I, m->p_xq, I, m->p_xs, st, false));
    }
    CK(lin(m->p_xq, I, Ld.down, EPI_RESID, m->p_x, D));
  }
  CK(launch_norm_q(m->p_x, D, m->gf, R, D, m->p_xq, D, m->p_xs, st, false, dig, nullptr, 0, Tpad));
  // head: unscaled per-group sums on the tensor cores, then the per-channel requant + argmax per row
  CK(lin(m->p_xq, D, m->head, EPI_RAW, m->p_raw, c.V));
  int64_t* lg = logits_host ? m->p_raw : nullptr;             // requant in place (row by row, read before write)
  CK(launch_head_rows(m->p_raw, c.V, R, m->head, m->p_xs, lg, c.V, m->p_next, st));
  if (logits_host) CK(cudaMemcpyAsync(logits_host, m->p_raw, sizeof(int64_t) * R * c.V, cudaMemcpyDeviceToHost, st));
  if (next_host) CK(cudaMemcpyAsync(next_host, m->p_next, sizeof(int32_t) * R, cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  return EXB_OK;
}

static bool prefill_tc_ok(exb_model* m) {
  const exb_config& c = m->c;
  if (m->tp > 1) return false;                 // tensor-parallel ranks run 4-row steps with in-graph collectives
  if (c.n_experts)
    return m->tc_on && !m->trace_on && !m->fr_on && gemm_tc_supported(m->L[0].qkv, EPI_RAW) &&
           gemm_tc_supported(m->L[0].o, EPI_RAW) && gemm_tc_supported(m->head, EPI_RAW) && c.D % 16 == 0;
  return m->tc_on && m->group && !m->trace_on && !m->fr_on && c.H * c.hd % 128 == 0 && gemm_tc_supported(m->L[0].qkv, EPI_STORE) &&
         gemm_tc_supported(m->L[0].gu, EPI_SWIGLU) && gemm_tc_supported(m->L[0].down, EPI_RESID) &&
         gemm_tc_supported(m->L[0].o, EPI_RESID) && gemm_tc_supported(m->head, EPI_RAW) && m->head.nodrop;
}

// logits of the R rows of the last step into host rows of the global vocabulary (tensor parallel:
// every rank's slice gathered with NCCL, then laid out in vocabulary order)
static int copy_logits(exb_model* m, int R, int64_t* host) {
  const int Vg = m->cg.V;
  if (m->tp == 1) {
    CK(cudaMemcpyAsync(host, m->logits, sizeof(int64_t) * R * Vg, cudaMemcpyDeviceToHost, m->st));
    return EXB_OK;
  }
  const size_t blk = (size_t)R * m->vmax;
  if (nccl()->all_gather(m->logits, m->tp_gather, blk, ncclInt64, m->comm, m->st) != ncclSuccess)
    FAIL(EXB_ECUDA, "ncclAllGather (logits) failed");
  std::vector<int64_t> g(blk * m->tp);
  CK(cudaMemcpyAsync(g.data(), m->tp_gather, sizeof(int64_t) * g.size(), cudaMemcpyDeviceToHost, m->st));
  CK(cudaStreamSynchronize(m->st));
  for (int k = 0; k < m->tp; ++k) {
    const int v0 = k * m->vmax, len = std::min(m->vmax, Vg - v0);
    for (int r = 0; r < R && len > 0; ++r)
      memcpy(host + (size_t)r * Vg + v0, g.data() + (size_t)k * blk + (size_t)r * m->vmax, sizeof(int64_t) * len);
  }
  return EXB_OK;
}

int exb_forward(exb_model* m, int n, const int32_t* ids, const int32_t* seqs, int64_t* logits, int32_t* next) {
  if (!m || !m->finalized) FAIL(EXB_EINVAL, "model not finalized");
  if (n <= 0 || !ids || !seqs) FAIL(EXB_EINVAL, "bad rows");
  const exb_config& c = m->c;
  std::vector<int> pos(n);
  std::vector<int> len = m->seq_len;
  for (int i = 0; i < n; ++i) {
    if (seqs[i] < 0 || seqs[i] >= c.max_batch) FAIL(EXB_EINVAL, "bad sequence slot");
    if (ids[i] < 0 || ids[i] >= m->cg.V) FAIL(EXB_EINVAL, "token id out of range");
    pos[i] = len[seqs[i]]++;
    if (pos[i] >= c.max_seq) FAIL(EXB_EINVAL, "sequence longer than max_seq");
  }
  if (m->trace_on) { m->trace_host.assign((size_t)n * m->trace_row, 0); m->trace_rows = n; }
  CK(cudaMemsetAsync(m->err, 0, sizeof(int), m->st));
  m->sel_rows = c.n_experts ? std::min(n, SEL_CAP) : 0;
  int r_tc = 0;                                              // rows done by tensor-core chunks
  if (n >= TC_MIN_ROWS && prefill_tc_ok(m)) {
    int rc = prefill_alloc(m);
    if (rc) return rc;
    while (n - r_tc >= TC_MIN_ROWS) {
      const int R = std::min(chunk_rows(m), n - r_tc);
      for (int r = 0; r < R; ++r) {
        m->p_hrows[r] = ids[r_tc + r]; m->p_hrows[PCH + r] = seqs[r_tc + r]; m->p_hrows[2 * PCH + r] = pos[r_tc + r];
      }
      g_hist_row0 = c.n_experts ? r_tc : -1;
      rc = prefill_chunk(m, R, logits ? logits + (size_t)r_tc * c.V : nullptr, next ? next + r_tc : nullptr);
      g_hist_row0 = -1;
      if (rc) return rc;
      r_tc += R;
    }
  }
  for (int r0 = r_tc; r0 < n; r0 += RMAX) {
    const int R = std::min(RMAX, n - r0);
    for (int r = 0; r < R; ++r) { m->h_ids[r] = ids[r0 + r]; m->h_seq[r] = seqs[r0 + r]; m->h_pos[r] = pos[r0 + r]; }
    CK(cudaMemcpyAsync(m->row_ids, m->h_ids, sizeof(int32_t) * RMAX * 3, cudaMemcpyHostToDevice, m->st));
    g_hist_row0 = c.n_experts ? r0 : -1;
    int rc = run_step(m, R, m->row_ids, m->row_seq, m->row_pos, logits != nullptr, 0);
    g_hist_row0 = -1;
    if (rc) return rc;
    if (logits) {
      rc = copy_logits(m, R, logits + (size_t)r0 * m->cg.V);
      if (rc) return rc;
    }
    if (next) CK(cudaMemcpyAsync(next + r0, m->next_tok, sizeof(int32_t) * R, cudaMemcpyDeviceToHost, m->st));
    if (m->trace_on)
      CK(cudaMemcpyAsync(m->trace_host.data() + (size_t)r0 * m->trace_row, m->trace, sizeof(int64_t) * R * m->trace_row,
                         cudaMemcpyDeviceToHost, m->st));
    if (m->fr_on) m->fr_checks += (int64_t)R * m->n_lin;
    // the pinned staging buffer is reused by the next chunk: wait for its copy
    CK(cudaStreamSynchronize(m->st));
  }
  m->seq_len = len;
  return check_device_errors(m);
}

// The token buffer holds max_batch x max_seq tokens (no call can produce more), allocated once:
// the captured generate graphs bake its address, so it must never move.
static int ensure_gen(exb_model* m, int B, int steps) {
  if (!m->gen_tokens) {
    const size_t cap = (size_t)m->c.max_batch * m->c.max_seq;
    CK(cudaMalloc(&m->gen_tokens, sizeof(int32_t) * cap));
    m->gen_cap = (int)cap;
  }
  if ((size_t)B * steps > (size_t)m->gen_cap) FAIL(EXB_EINVAL, "generate: more tokens than max_batch x max_seq");
  return EXB_OK;
}

// Greedy decode of B > 4 sequences: every step is one tensor-core chunk of B rows (row b = the
// last token of sequence b at its next position), next tokens fed back through the host.
static int generate_wide(exb_model* m, int B, const int32_t* ids_dev_or_null, const int32_t* ids_host, int steps,
                         int32_t* tokens_host, int64_t* logits_host, int32_t* tokens_dev) {
  const exb_config& c = m->c;
  if (B > chunk_rows(m) || !prefill_tc_ok(m))
    FAIL(EXB_EINVAL, "generate: B > 4 needs the tensor-core path and B <= 512 (256 for MoE)");
  int rc = prefill_alloc(m);
  if (rc) return rc;
  std::vector<int32_t> cur(B), nxt(B), toks((size_t)B * steps);
  if (ids_dev_or_null) CK(cudaMemcpy(cur.data(), ids_dev_or_null, 4 * (size_t)B, cudaMemcpyDeviceToHost));
  else memcpy(cur.data(), ids_host, 4 * (size_t)B);
  for (int b = 0; b < B; ++b)
    if (cur[b] < 0 || cur[b] >= m->cg.V) FAIL(EXB_EINVAL, "token id out of range");
  CK(cudaMemsetAsync(m->err, 0, sizeof(int), m->st));
  for (int s = 0; s < steps; ++s) {
    for (int b = 0; b < B; ++b) {
      m->p_hrows[b] = cur[b]; m->p_hrows[PCH + b] = b; m->p_hrows[2 * PCH + b] = m->seq_len[b] + s;
    }
    rc = prefill_chunk(m, B, logits_host ? logits_host + (size_t)s * B * c.V : nullptr, nxt.data());
    if (rc) return rc;
    for (int b = 0; b < B; ++b) toks[(size_t)s * B + b] = nxt[b];
    cur = nxt;
  }
  for (int b = 0; b < B; ++b) m->seq_len[b] += steps;
  if (tokens_host) memcpy(tokens_host, toks.data(), 4 * toks.size());
  if (tokens_dev) CK(cudaMemcpy(tokens_dev, toks.data(), 4 * toks.size(), cudaMemcpyHostToDevice));
  return check_device_errors(m);
}

static int generate_common(exb_model* m, int B, const int32_t* ids_dev_or_null, const int32_t* ids_host, int steps,
                           int32_t* tokens_host, int64_t* logits_host, int32_t* tokens_dev) {
  if (!m || !m->finalized) FAIL(EXB_EINVAL, "model not finalized");
  const exb_config& c = m->c;
  if (B <= 0 || B > c.max_batch) FAIL(EXB_EINVAL, "generate: 1 <= B <= max_batch");
  if (steps > 0)
    for (int b = 0; b < B; ++b)
      if (m->seq_len[b] + steps > c.max_seq) FAIL(EXB_EINVAL, "generate: max_seq exceeded");
  if (B > RMAX && steps > 0 && m->samp_on) FAIL(EXB_EINVAL, "generate: sampling runs batches of <= 4 rows");
  if (B > RMAX && steps > 0) return generate_wide(m, B, ids_dev_or_null, ids_host, steps, tokens_host, logits_host, tokens_dev);
  if (steps <= 0) return EXB_OK;
  struct SampScope {                    // sampling applies to these decode steps only
    exb_model* m;
    explicit SampScope(exb_model* mm) : m(mm) { m->samp_active = m->samp_on; }
    ~SampScope() { m->samp_active = false; }
  } samp_scope(m);
  for (int b = 0; b < B; ++b)
    if (m->seq_len[b] + steps > c.max_seq) FAIL(EXB_EINVAL, "generate: max_seq exceeded");
  int rc = ensure_gen(m, B, steps);
  if (rc) return rc;
  std::vector<int32_t> seq(B), pos(B);
  for (int b = 0; b < B; ++b) { seq[b] = b; pos[b] = m->seq_len[b]; }
  CK(cudaMemsetAsync(m->err, 0, sizeof(int), m->st));
  if (ids_dev_or_null) CK(cudaMemcpyAsync(m->gen_ids, ids_dev_or_null, 4 * B, cudaMemcpyDeviceToDevice, m->st));
  else CK(cudaMemcpyAsync(m->gen_ids, ids_host, 4 * B, cudaMemcpyHostToDevice, m->st));
  CK(cudaMemcpyAsync(m->gen_seq, seq.data(), 4 * B, cudaMemcpyHostToDevice, m->st));
  CK(cudaMemcpyAsync(m->gen_pos, pos.data(), 4 * B, cudaMemcpyHostToDevice, m->st));
  CK(cudaMemsetAsync(m->gen_step, 0, 4, m->st));
  if (m->trace_on) { m->trace_host.assign((size_t)B * steps * m->trace_row, 0); m->trace_rows = (int64_t)B * steps; }
  for (int s = 0; s < steps; ++s) {
    rc = run_step(m, B, m->gen_ids, m->gen_seq, m->gen_pos, logits_host != nullptr, B);
    if (rc) return rc;
    if (logits_host)
    {
      rc = copy_logits(m, B, logits_host + (size_t)s * B * m->cg.V);
      if (rc) return rc;
    }
    if (m->trace_on)
      CK(cudaMemcpyAsync(m->trace_host.data() + (size_t)s * B * m->trace_row, m->trace, sizeof(int64_t) * B * m->trace_row,
                         cudaMemcpyDeviceToHost, m->st));
    if (m->fr_on) m->fr_checks += (int64_t)B * m->n_lin;
  }
  if (tokens_dev) CK(cudaMemcpyAsync(tokens_dev, m->gen_tokens, sizeof(int32_t) * B * steps, cudaMemcpyDeviceToDevice, m->st));
  if (tokens_host) CK(cudaMemcpyAsync(tokens_host, m->gen_tokens, sizeof(int32_t) * B * steps, cudaMemcpyDeviceToHost, m->st));
  for (int b = 0; b < B; ++b) m->seq_len[b] += steps;
  if (tokens_host || logits_host || m->trace_on) return check_device_errors(m);
  return EXB_OK;
}

int exb_generate(exb_model* m, int B, const int32_t* first_ids, int steps, int32_t* tokens, int64_t* logits) {
  if (!first_ids || !tokens) FAIL(EXB_EINVAL, "null argument");
  return generate_common(m, B, nullptr, first_ids, steps, tokens, logits, nullptr);
}

int exb_generate_device(exb_model* m, int B, const int32_t* ids_dev, int steps, int32_t* tokens_dev) {
  if (!ids_dev || !tokens_dev) FAIL(EXB_EINVAL, "null argument");
  return generate_common(m, B, ids_dev, nullptr, steps, nullptr, nullptr, tokens_dev);
}

// KV cache of one layer and sequence slot, positions 0..n-1, as stored: K int16 (KV, n, hd) after
// RoPE and qrow, its per-row shift int8 (KV, n), V int32 (KV, n, hd) -- the reference cache's kq,
// sk and v (exact_torch.py:146-149).  Tensor parallel: this rank's KV heads.
int exb_kv_export(exb_model* m, int layer, int seq, int n, int16_t* k_host, int8_t* ks_host, int32_t* v_host) {
  if (!m || !m->finalized) FAIL(EXB_EINVAL, "model not finalized");
  const exb_config& c = m->c;
  if (layer < 0 || layer >= c.NL || seq < 0 || seq >= c.max_batch || n < 0 || n > c.max_seq)
    FAIL(EXB_EINVAL, "exb_kv_export: bad layer, sequence slot or position count");
  if (n > m->seq_len[seq]) FAIL(EXB_EINVAL, "exb_kv_export: the sequence holds fewer positions");
  if (n == 0) return EXB_OK;
  const size_t row0 = (size_t)seq * c.KV * c.max_seq;                  // (seq, head 0, position 0)
  const size_t lay = m->kv_layer_elems * layer, lay_s = (size_t)c.max_batch * c.KV * c.max_seq * layer;
  if (k_host)
    CK(cudaMemcpy2DAsync(k_host, sizeof(int16_t) * n * c.hd, m->kc + lay + row0 * c.hd, sizeof(int16_t) * c.max_seq * c.hd,
                         sizeof(int16_t) * n * c.hd, c.KV, cudaMemcpyDeviceToHost, m->st));
  if (v_host)
    CK(cudaMemcpy2DAsync(v_host, sizeof(int32_t) * n * c.hd, m->vc + lay + row0 * c.hd, sizeof(int32_t) * c.max_seq * c.hd,
                         sizeof(int32_t) * n * c.hd, c.KV, cudaMemcpyDeviceToHost, m->st));
  if (ks_host)
    CK(cudaMemcpy2DAsync(ks_host, n, m->ks + lay_s + row0, c.max_seq, n, c.KV, cudaMemcpyDeviceToHost, m->st));
  CK(cudaStreamSynchronize(m->st));
  return EXB_OK;
}

int exb_trace_enable(exb_model* m, int on) {
  if (!m) FAIL(EXB_EINVAL, "null model");
  if (on && m->c.n_experts) FAIL(EXB_EINVAL, "trace capture covers the dense models (the reference traces them only)");
  m->trace_on = on != 0;
  return EXB_OK;
}
int64_t exb_trace_row_len(exb_model* m) { return m ? (m->tp > 1 ? m->trace_row_g : m->trace_row) : -1; }
int exb_step_launches(exb_model* m) { return m ? m->step_kernels : -1; }
// ---- Merkle trace commitment
int exb_commit_begin(exb_model* m, int seq, int capacity) {
  if (!m || !m->finalized) FAIL(EXB_EINVAL, "exb_commit_begin: model not finalized");
  if (m->c.n_experts) FAIL(EXB_EINVAL, "exb_commit_begin: the commitment covers the dense models");
  if (m->tp > 1) FAIL(EXB_EINVAL, "exb_commit_begin: single-GPU models only");
  if (seq < 0 || seq >= m->c.max_batch || capacity < 1 || capacity > m->c.max_seq)
    FAIL(EXB_EINVAL, "exb_commit_begin: seq in [0, max_batch), capacity in [1, max_seq]");
  const size_t row = (size_t)(m->trace_row + m->cap_row);
  CK(cudaStreamSynchronize(m->st));
  cudaFree(m->commit_log);
  m->commit_log = nullptr;
  if (cudaMalloc(&m->commit_log, row * capacity * sizeof(int64_t)) != cudaSuccess) {
    cudaGetLastError();
    FAIL(EXB_ECUDA, "exb_commit_begin: no device memory for " + std::to_string(capacity) + " log rows of " +
                        std::to_string(row * 8) + " bytes");
  }
  if (!m->commit_lin) {
    std::vector<int64_t> h(2 * m->lins.size());
    for (size_t i = 0; i < m->lins.size(); ++i) {
      h[i] = m->lins[i].trace_off;
      h[m->lins.size() + i] = m->lins[i].N;
    }
    CK(cudaMalloc(&m->commit_lin, h.size() * sizeof(int64_t)));
    CK(cudaMemcpy(m->commit_lin, h.data(), h.size() * sizeof(int64_t), cudaMemcpyHostToDevice));
  }
  CK(cudaMemsetAsync(m->commit_npos, 0, sizeof(int), m->st));
  m->commit_on = true;
  m->trace_on = true;
  m->commit_seq = seq;
  m->commit_cap = capacity;
  for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
  m->graphs.clear();
  return EXB_OK;
}

int exb_commit_root(exb_model* m, int T, uint8_t* root32, uint8_t* leaves_host, int64_t leaves_bytes) {
  if (!m || !root32) FAIL(EXB_EINVAL, "null argument");
  if (!m->commit_on) FAIL(EXB_EINVAL, "exb_commit_root: call exb_commit_begin first");
  if (T < 1 || T > m->commit_cap) FAIL(EXB_EINVAL, "exb_commit_root: T in [1, capacity]");
  const exb_config& c = m->c;
  const int64_t n = commit_leaf_count(c.NL, T);
  if (leaves_host && leaves_bytes != n * 32)
    FAIL(EXB_EINVAL, "exb_commit_root: leaves buffer must hold " + std::to_string(n * 32) + " bytes");
  int npos = 0;
  CK(cudaMemcpyAsync(&npos, m->commit_npos, sizeof(int), cudaMemcpyDeviceToHost, m->st));
  CK(cudaStreamSynchronize(m->st));
  if (npos < T) FAIL(EXB_EINVAL, "exb_commit_root: only positions 0.." + std::to_string(npos - 1) + " were logged");
  CommitLayout L;
  L.NL = c.NL; L.D = c.D; L.KV = c.KV; L.hd = c.hd;
  L.x_off = m->trace_row;
  L.kr_off = m->trace_row + (int64_t)(c.NL + 1) * c.D;
  L.lin_off = m->commit_lin;
  L.lin_len = m->commit_lin + m->lins.size();
  uint8_t* buf = nullptr;
  const size_t lv = (size_t)n * 32;
  CK(cudaMalloc(&buf, 3 * lv));
  uint8_t* root_dev = nullptr;
  cudaError_t e = commit_root(m->commit_log, m->trace_row + m->cap_row, T, L, buf, buf + lv, buf + 2 * lv, &root_dev,
                              m->st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(root32, root_dev, 32, cudaMemcpyDeviceToHost, m->st);
  if (e == cudaSuccess && leaves_host) e = cudaMemcpyAsync(leaves_host, buf, lv, cudaMemcpyDeviceToHost, m->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->st);
  cudaFree(buf);
  if (e != cudaSuccess) FAIL(EXB_ECUDA, std::string("exb_commit_root: ") + cudaGetErrorString(e));
  return check_device_errors(m);
}

// ---- weightless cell verifier
int exb_verifier_emb_keys(exb_model* m, const int32_t* r_host) {
  if (!m || !m->finalized || !r_host) FAIL(EXB_EINVAL, "exb_verifier_emb_keys: null argument / not finalized");
  if (m->tp > 1) FAIL(EXB_EINVAL, "exb_verifier_emb_keys: single-GPU models");
  const exb_config& c = m->c;
  for (int i = 0; i < 2 * c.D; ++i)
    if (r_host[i] < 0 || (uint32_t)r_host[i] >= (i < c.D ? 2147483647u : 2147483629u))
      FAIL(EXB_EINVAL, "exb_verifier_emb_keys: r outside [0, p)");
  if (!m->ver_emb_r) CK(cudaMalloc(&m->ver_emb_r, sizeof(int32_t) * 2 * c.D));
  if (!m->ver_emb_de) CK(cudaMalloc(&m->ver_emb_de, sizeof(int64_t) * 2 * c.V));
  CK(cudaMemcpyAsync(m->ver_emb_r, r_host, sizeof(int32_t) * 2 * c.D, cudaMemcpyHostToDevice, m->st));
  CK(launch_emb_digest(m->emb, c.emb_shift, m->emb_q16, c.V, c.D, m->ver_emb_r, m->ver_emb_de, m->st));
  CK(cudaStreamSynchronize(m->st));
  return EXB_OK;
}

int exb_verify_cells(exb_model* m, int T, const uint8_t* root32, int n_cells, const int32_t* cells, const int32_t* ids,
                     const int64_t* values, int64_t n_values, const uint8_t* proofs, int64_t proof_bytes,
                     int32_t* verdicts) {
  if (!m || !m->finalized || !root32 || !cells || !ids || !values || !proofs || !verdicts)
    FAIL(EXB_EINVAL, "exb_verify_cells: null argument / not finalized");
  const exb_config& c = m->c;
  if (m->tp > 1 || c.n_experts) FAIL(EXB_EINVAL, "exb_verify_cells: dense single-GPU models");
  if (T < 1 || T > c.rope_len || n_cells < 1) FAIL(EXB_EINVAL, "exb_verify_cells: T in [1, rope_len], n_cells >= 1");
  for (auto& L : m->lins)
    if (!L.fr_d) FAIL(EXB_EINVAL, "exb_verify_cells: set the Freivalds keys first (exb_freivalds_set_keys)");
  if (!m->ver_emb_de) FAIL(EXB_EINVAL, "exb_verify_cells: set the embedding keys first (exb_verifier_emb_keys)");
  const int NL = c.NL, D = c.D, Hd = c.H * c.hd, KVd = c.KV * c.hd, I = c.I;
  const int64_t nleaves = commit_leaf_count(NL, T);
  int depth = 0;
  for (int64_t n = nleaves; n > 1; n = (n + 1) / 2) ++depth;
  // leaf records in needed() order (experiments/commit_audit_kaggle.py:647-651)
  std::vector<VLeafRec> recs;
  std::vector<int64_t> voff(n_cells);
  std::vector<int> leaf0(n_cells + 1);
  int64_t v = 0, pb = 0;
  auto lid = [&](int kind, int L, int t) -> int64_t {     // 0 X, 1 KV, 2 KR, 3 Q, 4 R, 5 HEAD
    if (kind == 0) return (int64_t)L * T + t;
    if (kind == 5) return (int64_t)(NL + 1) * T + 4ll * NL * T + t;
    return (int64_t)(NL + 1) * T + ((int64_t)L * T + t) * 4 + (kind - 1);
  };
  auto add = [&](int kind, int L, int t, std::initializer_list<int64_t> lens) {
    VLeafRec r;
    r.voff = v; r.leaf = lid(kind, L, t); r.poff = pb; r.nseg = (int)lens.size();
    int j = 0;
    for (int64_t x : lens) { r.len[j++] = x; v += x; }
    pb += 32ll * depth;
    recs.push_back(r);
  };
  for (int i = 0; i < n_cells; ++i) {
    const int L = cells[2 * i], t = cells[2 * i + 1];
    if (L < 0 || L > NL || t < 0 || t >= T) FAIL(EXB_EINVAL, "exb_verify_cells: cell outside (0..NL, 0..T-1)");
    voff[i] = v;
    leaf0[i] = (int)recs.size();
    if (L == NL) {
      add(0, NL, t, {D});
      add(5, NL, t, {c.V});
    } else {
      add(0, L, t, {D});
      add(1, L, t, {KVd, KVd});
      for (int s = 0; s <= t; ++s) add(2, L, s, {KVd, KVd});
      add(3, L, t, {Hd});
      add(4, L, t, {D, I, I, D});
      add(0, L + 1, t, {D});
    }
  }
  leaf0[n_cells] = (int)recs.size();
  if (v != n_values) FAIL(EXB_EINVAL, "exb_verify_cells: expected " + std::to_string(v) + " opened values");
  if (pb != proof_bytes) FAIL(EXB_EINVAL, "exb_verify_cells: expected " + std::to_string(pb) + " proof bytes");
  for (int t = 0; t < T; ++t)
    if (ids[t] < 0 || ids[t] >= c.V) FAIL(EXB_EINVAL, "exb_verify_cells: token id outside the vocabulary");
  // device copies
  std::vector<VLinDev> vl(m->lins.size());
  for (size_t i = 0; i < m->lins.size(); ++i) {
    const LinInfo& L = m->lins[i];
    VLinDev& d = vl[i];
    d.N = L.N; d.K = L.K; d.group = L.fused->Mg != nullptr; d.row0 = L.row0; d.row_step = L.row_step;
    d.mbits = L.mbits; d.b = L.fused->b; d.Mc = L.fused->Mc; d.r = L.fr_r; d.d = L.fr_d;
  }
  std::vector<const int64_t*> gains(2 * NL);
  for (int l = 0; l < NL; ++l) { gains[l] = m->L[l].g1; gains[NL + l] = m->L[l].g2; }
  const int ymax = std::max(std::max(I, Hd), 2 * KVd);
  const int q16 = std::max(std::max(D, Hd), I);
  const int64_t scr_len = 2ll * Hd + D + 2ll * ymax + (int64_t)c.H * T;
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t b_vl = al(vl.size() * sizeof(VLinDev)), b_g = al(gains.size() * 8), b_ids = al(4ull * T),
               b_cells = al(8ull * n_cells), b_val = al(8ull * v), b_voff = al(8ull * n_cells),
               b_l0 = al(4ull * (n_cells + 1)), b_rec = al(recs.size() * sizeof(VLeafRec)), b_pr = al(pb),
               b_root = al(32), b_ok = al(4 * recs.size() + 4), b_scr = al(8ull * scr_len * n_cells), b_vd = al(4ull * n_cells);
  char* buf = nullptr;
  const size_t total = b_vl + b_g + b_ids + b_cells + b_val + b_voff + b_l0 + b_rec + b_pr + b_root + b_ok + b_scr + b_vd;
  if (cudaMalloc(&buf, total) != cudaSuccess) {
    cudaGetLastError();
    FAIL(EXB_ECUDA, "exb_verify_cells: no device memory for " + std::to_string(total) + " bytes");
  }
  char* p = buf;
  auto take = [&](size_t b) { char* q = p; p += b; return q; };
  VLinDev* d_vl = (VLinDev*)take(b_vl);
  const int64_t** d_g = (const int64_t**)take(b_g);
  int32_t* d_ids = (int32_t*)take(b_ids);
  int32_t* d_cells = (int32_t*)take(b_cells);
  int64_t* d_val = (int64_t*)take(b_val);
  int64_t* d_voff = (int64_t*)take(b_voff);
  int* d_l0 = (int*)take(b_l0);
  VLeafRec* d_rec = (VLeafRec*)take(b_rec);
  uint8_t* d_pr = (uint8_t*)take(b_pr);
  uint8_t* d_root = (uint8_t*)take(b_root);
  int* d_ok = (int*)take(b_ok);
  int64_t* d_scr = (int64_t*)take(b_scr);
  int32_t* d_vd = (int32_t*)take(b_vd);
  cudaError_t e = cudaSuccess;
  auto up = [&](void* dst, const void* src, size_t b) {
    if (e == cudaSuccess && b) e = cudaMemcpyAsync(dst, src, b, cudaMemcpyHostToDevice, m->st);
  };
  up(d_vl, vl.data(), vl.size() * sizeof(VLinDev));
  up(d_g, gains.data(), gains.size() * 8);
  up(d_ids, ids, 4ull * T);
  up(d_cells, cells, 8ull * n_cells);
  up(d_val, values, 8ull * v);
  up(d_voff, voff.data(), 8ull * n_cells);
  up(d_l0, leaf0.data(), 4ull * (n_cells + 1));
  up(d_rec, recs.data(), recs.size() * sizeof(VLeafRec));
  up(d_pr, proofs, pb);
  up(d_root, root32, 32);
  VerifyArgs a;
  a.NL = NL; a.D = D; a.H = c.H; a.KV = c.KV; a.hd = c.hd; a.I = I; a.V = c.V; a.T = T;
  a.inv = (int64_t)std::nearbyint(65536.0 / std::sqrt((double)c.hd));
  a.lins = d_vl; a.g1 = d_g; a.g2 = d_g + NL; a.gf = m->gf;
  a.cos_t = m->cos_t; a.sin_t = m->sin_t; a.exp_t = m->exp_t; a.silu_t = m->silu_t;
  a.emb_r = m->ver_emb_r; a.emb_de = m->ver_emb_de; a.ids = d_ids; a.cells = d_cells;
  a.values = d_val; a.cell_voff = d_voff; a.cell_leaf0 = d_l0; a.leaf_ok = d_ok;
  a.scratch = d_scr; a.scr_len = scr_len; a.ymax = ymax; a.q16_len = q16; a.verdict = d_vd;
  if (e == cudaSuccess) e = launch_verify(a, n_cells, (int)recs.size(), d_rec, d_pr, depth, d_root, d_ok, m->st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(verdicts, d_vd, 4ull * n_cells, cudaMemcpyDeviceToHost, m->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->st);
  cudaFree(buf);
  if (e != cudaSuccess) FAIL(EXB_ECUDA, std::string("exb_verify_cells: ") + cudaGetErrorString(e));
  return check_device_errors(m);
}

// ---- integer sampler
int exb_sampling(exb_model* m, int on, int B, const uint64_t* seeds, const int32_t* positions, int64_t tnum) {
  if (!m || !m->finalized) FAIL(EXB_EINVAL, "exb_sampling: model not finalized");
  if (on) {
    if (m->tp > 1) FAIL(EXB_EINVAL, "exb_sampling: single-GPU models (the logits rows are sharded under TP)");
    if (B < 1 || B > RMAX || !seeds || !positions) FAIL(EXB_EINVAL, "exb_sampling: 1 <= B <= 4 rows of seeds and positions");
    if (tnum < 1 || tnum > (1ll << 32)) FAIL(EXB_EINVAL, "exb_sampling: temperature multiplier in [1, 2^32]");
    for (int b = 0; b < B; ++b)
      if (positions[b] < 0) FAIL(EXB_EINVAL, "exb_sampling: negative sampling position");
    CK(cudaMemcpyAsync(m->samp_seed, seeds, 8 * (size_t)B, cudaMemcpyHostToDevice, m->st));
    CK(cudaMemcpyAsync(m->samp_pos, positions, 4 * (size_t)B, cudaMemcpyHostToDevice, m->st));
    CK(cudaStreamSynchronize(m->st));
    m->samp_tnum = tnum;
  }
  m->samp_on = on != 0;
  return EXB_OK;
}

int exb_sampling_positions(exb_model* m, int32_t* positions, int B) {
  if (!m || !positions || B < 1 || B > RMAX) FAIL(EXB_EINVAL, "exb_sampling_positions: 1 <= B <= 4");
  CK(cudaMemcpyAsync(positions, m->samp_pos, 4 * (size_t)B, cudaMemcpyDeviceToHost, m->st));
  CK(cudaStreamSynchronize(m->st));
  return EXB_OK;
}

int exb_sample(exb_model* m, const int64_t* logits, int R, int V, const uint64_t* seeds, const int32_t* positions,
               int64_t tnum, int32_t* tokens) {
  if (!m || !m->finalized || !logits || !seeds || !positions || !tokens) FAIL(EXB_EINVAL, "exb_sample: null argument");
  if (R < 1 || V < 1 || tnum < 1 || tnum > (1ll << 32)) FAIL(EXB_EINVAL, "exb_sample: R >= 1, V >= 1, tnum in [1, 2^32]");
  for (int r = 0; r < R; ++r)
    if (positions[r] < 0) FAIL(EXB_EINVAL, "exb_sample: negative sampling position");
  const size_t lb = (size_t)R * V * 8;
  char* buf = nullptr;
  CK(cudaMalloc(&buf, lb + (size_t)R * 16));
  int64_t* dl = reinterpret_cast<int64_t*>(buf);
  unsigned long long* ds = reinterpret_cast<unsigned long long*>(buf + lb);
  int32_t* dp = reinterpret_cast<int32_t*>(buf + lb + (size_t)R * 8);
  int32_t* dt = dp + R;
  cudaError_t e = cudaMemcpyAsync(dl, logits, lb, cudaMemcpyHostToDevice, m->st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(ds, seeds, (size_t)R * 8, cudaMemcpyHostToDevice, m->st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dp, positions, (size_t)R * 4, cudaMemcpyHostToDevice, m->st);
  if (e == cudaSuccess) e = launch_sample(R, dl, V, V, ds, dp, false, tnum, m->exp_t, dt, m->st, false);
  if (e == cudaSuccess) e = cudaMemcpyAsync(tokens, dt, (size_t)R * 4, cudaMemcpyDeviceToHost, m->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->st);
  cudaFree(buf);
  if (e != cudaSuccess) FAIL(EXB_ECUDA, std::string("exb_sample: ") + cudaGetErrorString(e));
  return EXB_OK;
}

int exb_commit_end(exb_model* m) {
  if (!m) FAIL(EXB_EINVAL, "null model");
  CK(cudaStreamSynchronize(m->st));
  cudaFree(m->commit_log);
  m->commit_log = nullptr;
  m->commit_on = false;
  m->commit_cap = 0;
  for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
  m->graphs.clear();
  return EXB_OK;
}

// Tensor parallel: rank k's trace row, linear by linear, as (local offset, global offset, length)
// segments -- the same walk as plan_lins over rank k's slice of the architecture.
struct TraceSeg { int64_t loc, glob, n; };
static std::vector<TraceSeg> tp_trace_segs(const exb_config& g, int rank, int size) {
  int p[9];
  std::string why;
  std::vector<TraceSeg> out;
  if (!tp_plan(g, rank, size, p, why)) return out;
  const int64_t qn = (int64_t)(p[1] - p[0]) * g.hd, kn = (int64_t)(p[3] - p[2]) * g.hd, in = (int64_t)(p[5] - p[4]) * 128;
  const int64_t Q = (int64_t)g.H * g.hd, KVn = (int64_t)g.KV * g.hd;
  int64_t loc = 0, glob = 0;
  auto seg = [&](int64_t n_loc, int64_t col0, int64_t n_glob) {
    out.push_back({loc, glob + col0, n_loc});
    loc += n_loc; glob += n_glob;
  };
  for (int i = 0; i < g.NL; ++i) {
    seg(qn, (int64_t)p[0] * g.hd, Q);
    seg(kn, (int64_t)p[2] * g.hd, KVn);
    seg(kn, (int64_t)p[2] * g.hd, KVn);
    seg(g.D, 0, g.D);                                        // o: the full sum on every rank
    seg(in, (int64_t)p[4] * 128, g.I);
    seg(in, (int64_t)p[4] * 128, g.I);
    seg(g.D, 0, g.D);                                        // down
  }
  seg(p[7] - p[6], p[6], g.V);
  return out;
}

int exb_trace_read(exb_model* m, int64_t* host, int64_t n) {
  if (!m || !host) FAIL(EXB_EINVAL, "null argument");
  if (m->tp == 1) {
    const int64_t have = (int64_t)m->trace_host.size();
    if (n != have) FAIL(EXB_EINVAL, "trace size mismatch: expected " + std::to_string(have));
    memcpy(host, m->trace_host.data(), sizeof(int64_t) * n);
    return EXB_OK;
  }
  // collective: every rank's local rows (padded to the longest local row) are gathered with NCCL and
  // placed at their global columns
  const int64_t rows = m->trace_rows;
  if (n != rows * m->trace_row_g) FAIL(EXB_EINVAL, "trace size mismatch: expected " + std::to_string(rows * m->trace_row_g));
  std::vector<std::vector<TraceSeg>> segs(m->tp);
  int64_t lmax = 0;
  for (int k = 0; k < m->tp; ++k) {
    segs[k] = tp_trace_segs(m->cg, k, m->tp);
    if (segs[k].empty()) FAIL(EXB_EINVAL, "tensor-parallel plan failed");
    lmax = std::max(lmax, segs[k].back().loc + segs[k].back().n);
  }
  if (rows == 0) return EXB_OK;
  int64_t *src = nullptr, *dst = nullptr;
  CK(cudaMallocAsync(&src, sizeof(int64_t) * rows * lmax, m->st));
  CK(cudaMallocAsync(&dst, sizeof(int64_t) * rows * lmax * m->tp, m->st));
  std::vector<int64_t> all((size_t)rows * lmax * m->tp);
  CK(cudaMemcpy2DAsync(src, sizeof(int64_t) * lmax, m->trace_host.data(), sizeof(int64_t) * m->trace_row,
                       sizeof(int64_t) * m->trace_row, rows, cudaMemcpyHostToDevice, m->st));
  const bool ok = nccl()->all_gather(src, dst, (size_t)rows * lmax, ncclInt64, m->comm, m->st) == ncclSuccess;
  if (ok) CK(cudaMemcpyAsync(all.data(), dst, sizeof(int64_t) * all.size(), cudaMemcpyDeviceToHost, m->st));
  cudaFreeAsync(src, m->st);
  cudaFreeAsync(dst, m->st);
  CK(cudaStreamSynchronize(m->st));
  if (!ok) FAIL(EXB_ECUDA, "ncclAllGather (trace) failed");
  for (int k = 0; k < m->tp; ++k)
    for (int64_t r = 0; r < rows; ++r) {
      const int64_t* srow = all.data() + ((size_t)k * rows + r) * lmax;
      int64_t* drow = host + (size_t)r * m->trace_row_g;
      for (const TraceSeg& sg : segs[k]) memcpy(drow + sg.glob, srow + sg.loc, sizeof(int64_t) * sg.n);
    }
  return EXB_OK;
}

// Keys: r_host holds the GLOBAL r of every linear (2 x Ng, both primes).  Under tensor
// parallelism every rank checks its own shard exactly -- a column-split linear with the r of its
// own output columns (d over the full input), a row-split linear (o, down) on its partial sums
// with the full r (d over its input slice) -- so the kernels are the single-GPU ones and no check
// needs communication; exb_freivalds_read_keys reassembles the global d = (W M)^T r mod p.
int exb_freivalds_set_keys(exb_model* m, const int32_t* r_host, int64_t n) {
  if (!m || !r_host) FAIL(EXB_EINVAL, "null argument");
  int64_t need = 0;
  for (auto& L : m->lins) need += 2 * (int64_t)L.Ng;
  if (n != need) FAIL(EXB_EINVAL, "freivalds keys: expected " + std::to_string(need) + " r values");
  // key storage lives in the runtime arena's tail
  size_t off = (m->roff + 255) & ~size_t(255);
  int64_t pos = 0;
  unsigned long long* acc_base = m->fr_acc;
  int idx = 0;
  for (auto& L : m->lins) {
    L.fr_r = (int32_t*)(m->rarena + off); off += ((size_t)2 * L.N * 4 + 255) & ~size_t(255);
    L.fr_d = (int32_t*)(m->rarena + off); off += ((size_t)2 * L.K * 4 + 255) & ~size_t(255);
    if (off > m->rbytes) FAIL(EXB_ENOMEM, "freivalds key storage exhausted");
    const int c0 = L.col_split ? L.r_lo : 0;                 // this rank's rows of the global r
    for (int p = 0; p < 2; ++p)
      CK(cudaMemcpyAsync(L.fr_r + (size_t)p * L.N, r_host + pos + (size_t)p * L.Ng + c0, sizeof(int32_t) * L.N,
                         cudaMemcpyHostToDevice, m->st));
    pos += 2 * (int64_t)L.Ng;
    const LinW& F = *L.fused;
    CK(launch_fr_keys(F.w, F.Mg, F.ldm, L.N, L.K, L.row0, L.row_step, L.fr_r, L.fr_d, m->st));
    L.fr_acc = acc_base + (size_t)idx * RMAX * 4;
    ++idx;
  }
  CK(cudaStreamSynchronize(m->st));
  for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
  m->graphs.clear();
  return EXB_OK;
}

static constexpr int64_t FR_P1 = 2147483647, FR_P2 = 2147483629;

int exb_freivalds_read_keys(exb_model* m, int32_t* d_host, int64_t n) {
  if (!m || !d_host) FAIL(EXB_EINVAL, "null argument");
  int64_t need = 0;
  for (auto& L : m->lins) need += 2 * (int64_t)L.Kg;
  if (n != need) FAIL(EXB_EINVAL, "freivalds read: expected " + std::to_string(need));
  for (auto& L : m->lins)
    if (!L.fr_d) FAIL(EXB_EINVAL, "keys not set");
  if (m->tp == 1) {
    int64_t pos = 0;
    for (auto& L : m->lins) {
      CK(cudaMemcpy(d_host + pos, L.fr_d, sizeof(int32_t) * 2 * L.K, cudaMemcpyDeviceToHost));
      pos += 2 * L.K;
    }
    return EXB_OK;
  }
  // collective: each rank's share of the global d (column-split: d over the full input, counted once
  // per distinct slice; row-split: d of its input columns), summed over the ranks with NCCL, mod p
  std::vector<int64_t> part((size_t)n, 0);
  int64_t pos = 0;
  std::vector<int32_t> d;
  for (auto& L : m->lins) {
    d.resize((size_t)2 * L.K);
    CK(cudaMemcpy(d.data(), L.fr_d, sizeof(int32_t) * 2 * L.K, cudaMemcpyDeviceToHost));
    if (L.col_split ? L.kv_owner : true) {
      const int k0 = L.col_split ? 0 : L.c_lo;
      for (int p = 0; p < 2; ++p)
        for (int k = 0; k < L.K; ++k) part[pos + (size_t)p * L.Kg + k0 + k] = d[(size_t)p * L.K + k];
    }
    pos += 2 * (int64_t)L.Kg;
  }
  int64_t* buf = nullptr;
  CK(cudaMallocAsync(&buf, sizeof(int64_t) * n, m->st));
  CK(cudaMemcpyAsync(buf, part.data(), sizeof(int64_t) * n, cudaMemcpyHostToDevice, m->st));
  const bool ok = nccl()->all_reduce(buf, buf, (size_t)n, ncclInt64, ncclSum, m->comm, m->st) == ncclSuccess;
  if (ok) CK(cudaMemcpyAsync(part.data(), buf, sizeof(int64_t) * n, cudaMemcpyDeviceToHost, m->st));
  cudaFreeAsync(buf, m->st);
  CK(cudaStreamSynchronize(m->st));
  if (!ok) FAIL(EXB_ECUDA, "ncclAllReduce (Freivalds keys) failed");
  pos = 0;
  for (auto& L : m->lins) {
    for (int p = 0; p < 2; ++p)
      for (int k = 0; k < L.Kg; ++k)
        d_host[pos + (size_t)p * L.Kg + k] = (int32_t)(part[pos + (size_t)p * L.Kg + k] % (p ? FR_P2 : FR_P1));
    pos += 2 * (int64_t)L.Kg;
  }
  return EXB_OK;
}

int exb_freivalds_enable(exb_model* m, int on) {
  if (!m) FAIL(EXB_EINVAL, "null model");
  if (on && (m->lins.empty() || !m->lins[0].fr_r)) FAIL(EXB_EINVAL, "set keys first");
  m->fr_on = on != 0;
  if (on) { CK(cudaMemset(m->fr_fail, 0, sizeof(int))); m->fr_checks = 0; }
  return EXB_OK;
}

int exb_freivalds_status(exb_model* m, int64_t* checks, int64_t* failures) {
  if (!m) FAIL(EXB_EINVAL, "null model");
  int f = 0;
  CK(cudaStreamSynchronize(m->st));
  CK(cudaMemcpy(&f, m->fr_fail, sizeof(int), cudaMemcpyDeviceToHost));
  int64_t v[2] = {m->fr_checks, f};
  if (m->tp > 1) {
    // collective: totals over the ranks (each rank checks its own shard)
    int64_t* buf = nullptr;
    CK(cudaMallocAsync(&buf, sizeof v, m->st));
    CK(cudaMemcpyAsync(buf, v, sizeof v, cudaMemcpyHostToDevice, m->st));
    const bool ok = nccl()->all_reduce(buf, buf, 2, ncclInt64, ncclSum, m->comm, m->st) == ncclSuccess;
    if (ok) CK(cudaMemcpyAsync(v, buf, sizeof v, cudaMemcpyDeviceToHost, m->st));
    cudaFreeAsync(buf, m->st);
    CK(cudaStreamSynchronize(m->st));
    if (!ok) FAIL(EXB_ECUDA, "ncclAllReduce (Freivalds status) failed");
  }
  if (checks) *checks = v[0];
  if (failures) *failures = v[1];
  return EXB_OK;
}

int exb_set_option(exb_model* m, const char* name, int64_t value) {
  if (!m || !name) FAIL(EXB_EINVAL, "null argument");
  const std::string n(name);
  if (n == "tc") m->tc_on = value != 0;
  else if (n == "fuse") m->fuse_in = (int)value;
  else if (n == "tpar") m->tpar = value != 0;
  else if (n == "tpx") m->tpx_opt = value != 0;
  else if (n == "tcp") gemm_tc_set_persist(value != 0 ? 1 : 0);
  else if (n == "tail") m->tail_norm = value != 0;

  else if (n == "attn") m->attn_fused = value != 0;
  else if (n == "pattn") m->attn_prefill = value != 0;
  else if (n == "tcd") m->tc_decode = value != 0;
  else FAIL(EXB_EINVAL, "unknown option " + n);
  CK(cudaStreamSynchronize(m->st));
  for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
  m->graphs.clear();
  return EXB_OK;
}

int exb_moe_selections(exb_model* m, int layer, int32_t* host, int64_t n) {
  if (!m || !host || !m->c.n_experts || layer < 0 || layer >= m->c.NL) FAIL(EXB_EINVAL, "exb_moe_selections: bad arguments");
  const int64_t need = m->sel_rows * m->c.topk;
  if (n != need) FAIL(EXB_EINVAL, "exb_moe_selections: expected " + std::to_string(need) + " values");
  CK(cudaStreamSynchronize(m->st));
  CK(cudaMemcpy(host, m->moe_hist + (size_t)layer * SEL_CAP * m->c.topk, sizeof(int32_t) * need, cudaMemcpyDeviceToHost));
  return EXB_OK;
}

#ifdef EXB_TIMELINE
// Timeline build only: op 0 installs a zeroed stamp buffer in every translation unit, op 1
// resets it, op 2 copies n x 8 stamps (see TlBuf) to `host`.
int exb_timeline(int op, uint64_t* host, int n) {
  static TlBuf* buf = nullptr;
  if (op == 0 && !buf) {
    if (cudaMalloc(&buf, sizeof(TlBuf)) != cudaSuccess) FAIL(EXB_ECUDA, "timeline alloc");
    for (auto fn : tl_installers())
      if (fn(buf)) FAIL(EXB_ECUDA, "timeline install");
  }
  if (!buf) FAIL(EXB_EINVAL, "timeline not installed");
  if (op <= 1) {
    std::vector<unsigned long long> h(sizeof(TlBuf) / 8, 0);
    for (int i = 0; i < TL_SLOTS; ++i) h[4 + 8 * i] = h[5 + 8 * i] = h[10 + 8 * i] = ~0ull;
    for (int i = 0; i < TL_SLOTS; ++i)
      for (int f = 0; f < 8; ++f) h[4 + 8 * TL_SLOTS + 16 * i + f] = ~0ull;
    CK(cudaMemcpy(buf, h.data(), sizeof(TlBuf), cudaMemcpyHostToDevice));
    return EXB_OK;
  }
  if (n > TL_SLOTS) n = TL_SLOTS;
  CK(cudaMemcpy(host, reinterpret_cast<char*>(buf) + 32, (size_t)n * 64, cudaMemcpyDeviceToHost));
  if (op == 3)   // in-kernel points follow the stamps in `host`
    CK(cudaMemcpy(host + (size_t)n * 8, reinterpret_cast<char*>(buf) + 32 + (size_t)TL_SLOTS * 64, (size_t)n * 128,
                  cudaMemcpyDeviceToHost));
  return EXB_OK;
}
#endif

int exb_device_errors(exb_model* m, int* bits) {
  if (!m || !bits) FAIL(EXB_EINVAL, "null argument");
  CK(cudaStreamSynchronize(m->st));
  CK(cudaMemcpy(bits, m->err, sizeof(int), cudaMemcpyDeviceToHost));
  return EXB_OK;
}

int exb_bench_linear(exb_model* m, int layer, int which, int R, int reps, float* avg_ms, double* bytes) {
  if (!m || !m->finalized || layer < 0 || layer >= m->c.NL || which < 0 || which > 4 || R < 1 || R > RMAX || reps < 1)
    FAIL(EXB_EINVAL, "exb_bench_linear: bad arguments");
  LayerDev& Ld = m->L[layer];
  GemvArgs g;
  g.xq = m->xq; g.xs = m->xs; g.ldx = m->KMAX; g.R = R; g.err = m->err;
  const exb_config& c = m->c;
  switch (which) {
    case 0: g.L = Ld.qkv; g.epi = EPI_STORE; g.out = m->qkv; g.ldo = m->Nqkv; break;
    case 1: g.L = Ld.o; g.epi = EPI_RESID; g.out = m->x; g.ldo = c.D; break;
    case 2: g.L = Ld.gu; g.epi = EPI_SWIGLU; g.out = m->hb; g.ldo = c.I; g.silu_t = m->silu_t; break;
    case 3: g.L = Ld.down; g.epi = EPI_RESID; g.out = m->x; g.ldo = c.D; break;
    default:
      g.L = m->head; g.epi = EPI_HEAD; g.out = nullptr; g.head_part = m->head_part; g.head_ticket = m->head_ticket;
      g.next_tok = m->next_tok; g.grid = m->head_grid; break;
  }
  // keep the activations in range: zero input rows (timing does not depend on values)
  CK(cudaMemsetAsync(m->xq, 0, sizeof(int16_t) * (size_t)RMAX * m->KMAX, m->st));
  CK(cudaMemsetAsync(m->xs, 0, sizeof(int32_t) * RMAX, m->st));
  cudaEvent_t e0, e1;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  CK(launch_gemv(g, m->st, false));  // warm-up
  CK(cudaEventRecord(e0, m->st));
  for (int i = 0; i < reps; ++i) CK(launch_gemv(g, m->st, false));
  CK(cudaEventRecord(e1, m->st));
  CK(cudaEventSynchronize(e1));
  float ms = 0;
  CK(cudaEventElapsedTime(&ms, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (avg_ms) *avg_ms = ms / reps;
  if (bytes) {
    const LinW& L = g.L;
    double b = (double)L.N * L.K + (L.Mg ? 4.0 * L.N * (L.K / 128) : 8.0 * L.N) + (L.b ? 8.0 * L.N : 0) +
               2.0 * R * L.K;
    const int nout = which == 2 ? L.N / 2 : (which == 4 ? 0 : L.N);
    b += 8.0 * R * nout * ((which == 1 || which == 3) ? 2 : 1);   // residual: read + write
    *bytes = b;
  }
  return EXB_OK;
}

int exb_profile_step(exb_model* m, int B, float* ms_out, int max_n, int* n_out) {
  if (!m || !m->finalized || B < 1 || B > RMAX || !ms_out || !n_out) FAIL(EXB_EINVAL, "exb_profile_step: bad arguments");
  std::vector<int32_t> h(3 * RMAX, 0);
  for (int b = 0; b < B; ++b) { h[b] = 0; h[RMAX + b] = b; h[2 * RMAX + b] = m->seq_len[b]; }
  for (int b = 0; b < B; ++b)
    if (m->seq_len[b] >= m->c.max_seq) FAIL(EXB_EINVAL, "exb_profile_step: sequence full");
  CK(cudaMemcpyAsync(m->row_ids, h.data(), sizeof(int32_t) * 3 * RMAX, cudaMemcpyHostToDevice, m->st));
  std::vector<cudaEvent_t> evs;
  cudaEvent_t e0;
  CK(cudaEventCreate(&e0));
  CK(cudaEventRecord(e0, m->st));
  g_prof = &evs;
  cudaError_t e = enqueue_step(m, B, m->row_ids, m->row_seq, m->row_pos, false, m->st);
  g_prof = nullptr;
  CK(cudaStreamSynchronize(m->st));
  int n = 0;
  cudaEvent_t prev = e0;
  for (auto ev : evs) {
    float ms = 0;
    cudaEventElapsedTime(&ms, prev, ev);
    if (n < max_n) ms_out[n] = ms;
    ++n;
    if (prev != e0) cudaEventDestroy(prev);
    prev = ev;
  }
  if (prev != e0) cudaEventDestroy(prev);
  cudaEventDestroy(e0);
  *n_out = n;
  if (e != cudaSuccess) FAIL(EXB_ECUDA, std::string("profile step: ") + cudaGetErrorString(e));
  return check_device_errors(m);   // the step wrote position seq_len (not advanced): harmless
}

void* exb_model_stream(exb_model* m) { return m ? (void*)m->st : nullptr; }
size_t exb_model_weight_bytes(exb_model* m) { return m ? m->wbytes : 0; }

}  // extern "C"
