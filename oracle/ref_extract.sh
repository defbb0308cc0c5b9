#!/bin/sh
# Test infrastructure: copies the reference's own host code for the cache path
# out of its engine source into oracle/_ref/ (git-ignored) so that
# ref_harness.cpp can compile it unchanged.  Nothing extracted is committed.
# Each range is checked against a marker on its first and last line, so a
# different reference revision fails here instead of compiling the wrong code.
#   usage: ref_extract.sh <reference src dir> <output dir>
set -eu
SRC="$1/engine.cpp"
OUT="$2"
mkdir -p "$OUT"

take() {  # name first last first-marker last-marker
    name=$1; a=$2; b=$3
    sed -n "${a}p" "$SRC" | grep -qF -- "$4" || { echo "ref_extract: $name: line $a lacks '$4'" >&2; exit 1; }
    sed -n "${b}p" "$SRC" | grep -qF -- "$5" || { echo "ref_extract: $name: line $b lacks '$5'" >&2; exit 1; }
    { echo "// engine.cpp:$a-$b"; sed -n "${a},${b}p" "$SRC"; } > "$OUT/$name.inc"
}

# file-scope state: KV caches, DeltaNet/conv state, cached tokens (engine.cpp:82-97)
take globals        82   97 'kv_dim'                        'g_cached_tokens'
# per-step timers the hot blocks add to (engine.cpp:3078-3082)
take timers       3078 3082 'g_time_gemv'                   'g_time_tp_reduce'
# the 4-thread pool the DeltaNet heads run on (engine.cpp:1630-1693)
take worker_pool  1630 1693 'struct WorkerPool'             'static WorkerPool g_worker_pool'
# Schraudolph exp, sigmoid, SiLU, AVX-512 SiLU (engine.cpp:2347-2376)
take fast_math    2347 2376 "Schraudolph's method"          '}'
# decode scratch vectors (engine.cpp:2381-2399)
take scratch      2381 2399 'g_norm_out'                    'g_logits'
# RoPE table and rotation (engine.cpp:2405-2432)
take rope         2405 2432 'g_rope_cos'                    '}'
# DeltaNet decode: conv + SiLU, split, norms, decay/beta, delta rule, gated RMSNorm
take gdn_decode   3198 3330 'auto t_host0'                  'g_time_host'
# attention decode: de-interleave, Q/K RMSNorm, RoPE, append, online softmax, gate
take attn_decode  3484 3566 'auto t_host1'                  'g_time_host'
# prefix rule of generate() (engine.cpp:4059-4077)
take prefix_rule  4059 4077 'int prefix_len = 0'            '}'
# reset_state (engine.cpp:4164-4176)
take reset_state  4164 4176 'void reset_state()'            '}'
