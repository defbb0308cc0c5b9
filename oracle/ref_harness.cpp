// TEST INFRASTRUCTURE ONLY — never linked, loaded or run by the product.
//
// Harness that compiles the reference's own host code for the per-token cache
// path (blocks of src/engine.cpp, copied unchanged into oracle/_ref/*.inc by
// ref_extract.sh at build time; nothing of it is committed) into
// oracle/_ref/libref.so, so that the oracle restatement (oracle.cpp) and the
// committed golden fixtures can be pinned to what the reference computes.
//
// The reference's engine.cpp cannot be compiled whole here (it needs
// tt-metalium and clang++-20).  The cache-path blocks themselves only use
// the standard library, libm and AVX-512F intrinsics, so this file supplies
// the few names they expect from the surrounding function bodies:
//   - `lw` (the DeltaNet layer's host weights, src/engine.h:45-50),
//   - `aw` (SmallAttnWeights, src/engine.cpp:1769-1772),
//   - `ssm_idx`, `attn_idx`, `pos`, `qkv`, `q_dim`, `kv_dim_one`
//     (src/engine.cpp:3445-3447), `Clock` (src/engine.cpp:3085),
//   - `g_pos`, `g_hidden_f32` (src/engine.cpp:70,79) for reset_state.
// and runs each block on caller-provided inputs.  Build flags follow the
// reference's engine build (Makefile: -O3 -std=gnu++20 -ffast-math, -march
// native; here x86-64-v4 so the library runs on any AVX-512 host), with g++ in
// place of clang++-20, which is absent.
#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cfloat>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "model_config.h"

using MC = ModelConfig;

static int g_pos = 0;
static std::vector<float> g_hidden_f32(MC::n_embd);

#include "globals.inc"
#include "timers.inc"
#include "worker_pool.inc"
#include "fast_math.inc"
#include "scratch.inc"
#include "rope.inc"
#include "reset_state.inc"

namespace {

struct GdnHostWeights {  // the fields of the reference's layer weights the block reads
  std::vector<float> ssm_conv1d_host, ssm_a_host, ssm_dt_bias_host, ssm_norm_host;
};
struct AttnHostWeights {
  std::vector<float> q_norm, k_norm;
};

std::once_flag g_started;
std::mutex g_call;  // the blocks use file-scope state: one call at a time
int g_rope_ctx = 0;

void start_pool() {
  std::call_once(g_started, [] {
    g_worker_pool.start();
    std::atexit([] { g_worker_pool.stop(); });
  });
}

void ensure_rope(int need) {
  if (need > g_rope_ctx) {
    need = std::max(need, 2 * g_rope_ctx);  // table rows do not depend on its length
    precompute_rope(need);
    g_rope_ctx = need;
  }
}

}  // namespace

extern "C" {

// One DeltaNet decode step of one layer (src/engine.cpp:3198-3330).
//   proj      [12352] f32: conv inputs | z | alpha | beta
//   conv      [3][8192] f32 conv history, shifted in place
//   state     [32][128][128] f32, updated in place
//   conv_w_t  [4][8192] f32 (the loader's transposed layout, gguf_loader.cpp:389-396)
//   out       [4096] f32: gated-RMSNorm output
void ref_gdn_decode(const float* proj, float* conv, float* state, const float* conv_w_t,
                    const float* ssm_a, const float* dt_bias, const float* ssm_norm, float* out) {
  start_pool();
  std::lock_guard<std::mutex> lk(g_call);
  using Clock = std::chrono::high_resolution_clock;
  const int ssm_idx = 0;
  GdnHostWeights lw;
  lw.ssm_conv1d_host.assign(conv_w_t, conv_w_t + 4 * MC::ssm_conv_channels);
  lw.ssm_a_host.assign(ssm_a, ssm_a + MC::ssm_dt_rank);
  lw.ssm_dt_bias_host.assign(dt_bias, dt_bias + MC::ssm_dt_rank);
  lw.ssm_norm_host.assign(ssm_norm, ssm_norm + MC::ssm_head_v_dim);
  const size_t ns = (size_t)ssm_n_v_heads * ssm_head_k_dim * ssm_head_v_dim_c;
  g_ssm_state[0].assign(state, state + ns);
  g_conv_state[0].assign(conv, conv + (size_t)conv_state_len * MC::ssm_conv_channels);
  std::memcpy(g_proj.data(), proj, sizeof(float) * g_combined_rows);
  {
#include "gdn_decode.inc"
  }
  std::memcpy(state, g_ssm_state[0].data(), sizeof(float) * ns);
  std::memcpy(conv, g_conv_state[0].data(),
              sizeof(float) * conv_state_len * MC::ssm_conv_channels);
  std::memcpy(out, g_ssm_proj_in.data(), sizeof(float) * MC::ssm_d_inner);
}

// One attention decode step of one layer at position `pos_in`
// (src/engine.cpp:3484-3566).
//   qkv      [10240] f32 projection row ([16][q|gate], k [4][256], v [4][256])
//   k_cache, v_cache  [pos_in + 1][4][256] f32; row pos_in is written (the append)
//   out      [4096] f32: gated attention output
void ref_attn_decode(const float* qkv_in, const float* q_norm, const float* k_norm, int pos_in,
                     float* k_cache, float* v_cache, float* out) {
  std::lock_guard<std::mutex> lk(g_call);
  using Clock = std::chrono::high_resolution_clock;
  const int attn_idx = 0;
  const int pos = pos_in;
  ensure_rope(pos + 1);
  AttnHostWeights aw;
  aw.q_norm.assign(q_norm, q_norm + MC::head_dim);
  aw.k_norm.assign(k_norm, k_norm + MC::head_dim);
  const size_t rows = (size_t)(pos + 1) * kv_dim;
  g_k_cache[0].assign(k_cache, k_cache + rows);
  g_v_cache[0].assign(v_cache, v_cache + rows);
  constexpr int q_dim = MC::n_head * MC::head_dim * 2;
  constexpr int kv_dim_one = MC::n_head_kv * MC::head_dim;
  float* qkv = g_qkv.data();
  std::memcpy(qkv, qkv_in, sizeof(float) * g_qkv_rows);
  {
#include "attn_decode.inc"
  }
  std::memcpy(k_cache + (size_t)pos * kv_dim, g_k_cache[0].data() + (size_t)pos * kv_dim,
              sizeof(float) * kv_dim);
  std::memcpy(v_cache + (size_t)pos * kv_dim, g_v_cache[0].data() + (size_t)pos * kv_dim,
              sizeof(float) * kv_dim);
  std::memcpy(out, g_attn_out.data(), sizeof(float) * MC::n_head * MC::head_dim);
}

// Resident variants for timing the reference: the caches and state stay in
// the reference's own file-scope vectors between calls, as in the engine, so
// a timed call does only the work of the cited block.
//   ref_set_layer: stands up attention cache `attn_idx` (< 8) with rows
//     [0, n) of k/v ([n][4][256] f32, capacity cap rows) and DeltaNet slot
//     `ssm_idx` (< 24) with state and conv history (either part may be NULL).
void ref_set_layer(int attn_idx, const float* k, const float* v, int n, int cap, int ssm_idx,
                   const float* state, const float* conv) {
  std::lock_guard<std::mutex> lk(g_call);
  if (k && v && attn_idx >= 0 && attn_idx < 8) {
    g_k_cache[attn_idx].assign((size_t)cap * kv_dim, 0.0f);
    g_v_cache[attn_idx].assign((size_t)cap * kv_dim, 0.0f);
    std::memcpy(g_k_cache[attn_idx].data(), k, sizeof(float) * n * kv_dim);
    std::memcpy(g_v_cache[attn_idx].data(), v, sizeof(float) * n * kv_dim);
  }
  if (state && conv && ssm_idx >= 0 && ssm_idx < 24) {
    const size_t ns = (size_t)ssm_n_v_heads * ssm_head_k_dim * ssm_head_v_dim_c;
    g_ssm_state[ssm_idx].assign(state, state + ns);
    g_conv_state[ssm_idx].assign(conv, conv + (size_t)conv_state_len * MC::ssm_conv_channels);
  }
}

// The DeltaNet block on resident slot `ssm_idx_in`; weights as in ref_gdn_decode.
void ref_gdn_decode_resident(int ssm_idx_in, const float* proj, const float* conv_w_t,
                             const float* ssm_a, const float* dt_bias, const float* ssm_norm,
                             float* out) {
  start_pool();
  std::lock_guard<std::mutex> lk(g_call);
  using Clock = std::chrono::high_resolution_clock;
  const int ssm_idx = ssm_idx_in;
  static GdnHostWeights lw;  // the engine keeps them resident too
  lw.ssm_conv1d_host.assign(conv_w_t, conv_w_t + 4 * MC::ssm_conv_channels);
  lw.ssm_a_host.assign(ssm_a, ssm_a + MC::ssm_dt_rank);
  lw.ssm_dt_bias_host.assign(dt_bias, dt_bias + MC::ssm_dt_rank);
  lw.ssm_norm_host.assign(ssm_norm, ssm_norm + MC::ssm_head_v_dim);
  std::memcpy(g_proj.data(), proj, sizeof(float) * g_combined_rows);
  {
#include "gdn_decode.inc"
  }
  std::memcpy(out, g_ssm_proj_in.data(), sizeof(float) * MC::ssm_d_inner);
}

// The attention block on resident cache `attn_idx_in` at position pos_in
// (capacity must exceed pos_in).
void ref_attn_decode_resident(int attn_idx_in, const float* qkv_in, const float* q_norm,
                              const float* k_norm, int pos_in, float* out) {
  std::lock_guard<std::mutex> lk(g_call);
  using Clock = std::chrono::high_resolution_clock;
  const int attn_idx = attn_idx_in;
  const int pos = pos_in;
  ensure_rope(pos + 1);
  AttnHostWeights aw;
  aw.q_norm.assign(q_norm, q_norm + MC::head_dim);
  aw.k_norm.assign(k_norm, k_norm + MC::head_dim);
  constexpr int q_dim = MC::n_head * MC::head_dim * 2;
  constexpr int kv_dim_one = MC::n_head_kv * MC::head_dim;
  float* qkv = g_qkv.data();
  std::memcpy(qkv, qkv_in, sizeof(float) * g_qkv_rows);
  {
#include "attn_decode.inc"
  }
  std::memcpy(out, g_attn_out.data(), sizeof(float) * MC::n_head * MC::head_dim);
}

// The prefix rule of generate() (src/engine.cpp:4059-4077) against a cached
// token list.  Returns the reused prefix length; *resets = how many times the
// block called reset_state() (0 or 1).
int ref_prefix_rule(const int32_t* cached, int n_cached, const int32_t* prompt, int n_prompt,
                    int* resets) {
  std::lock_guard<std::mutex> lk(g_call);
  g_cached_tokens.assign(cached, cached + n_cached);
  std::vector<int> tokens(prompt, prompt + n_prompt);
  g_pos = -1;  // reset_state() sets it to 0
  {
#include "prefix_rule.inc"
    *resets = g_pos == 0 ? 1 : 0;
    return prefix_len;
  }
}

// cos/sin of the reference's RoPE table at one position (src/engine.cpp:2408-2420).
void ref_rope_row(int pos, float* cos_out, float* sin_out) {
  std::lock_guard<std::mutex> lk(g_call);
  ensure_rope(pos + 1);
  constexpr int half = MC::rope_dim / 2;
  std::memcpy(cos_out, g_rope_cos.data() + (size_t)pos * half, sizeof(float) * half);
  std::memcpy(sin_out, g_rope_sin.data() + (size_t)pos * half, sizeof(float) * half);
}

float ref_fast_expf(float x) { return fast_expf(x); }

}  // extern "C"
