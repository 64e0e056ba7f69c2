#!/usr/bin/env bash
# Builds the oracle libraries (test infrastructure only):
#   oracle/liboracle.so    the C restatement (oracle.c), gcc, OpenMP;
#   oracle/_ref/libref.so  the reference's own sources, compiled unchanged from where they
#                          lie (REF: the reference checkout's root): its CPU attention harness and
#                          its K10-K15 CUDA kernels for sm_100a;
#   oracle/_ref/libref_engine.so  the reference's GPT2Engine (src/gpt2_engine.cu, sampler, the
#                          kernels it calls) with a C entry that runs greedy generation.
# Both are skipped when REF is absent (the GPU box uses the prebuilt files).
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
REF="${REF:-/root/reference}"
NVCC="${NVCC:-/usr/local/cuda/bin/nvcc}"
gcc -O2 -fPIC -shared -fopenmp -ffp-contract=off -o "$HERE/liboracle.so" "$HERE/oracle.c" -lm
if [ -d "$REF/kernels" ]; then
  mkdir -p "$HERE/_ref"
  "$NVCC" -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -shared -Xcompiler -fPIC \
    -Xcompiler -fvisibility=hidden -Xcompiler -ffp-contract=off \
    -I "$HERE/ref_shim" -I "$REF/include" -I "$REF/kernels" -I "$REF" \
    -o "$HERE/_ref/libref.so" \
    "$HERE/ref_wrappers.cu" \
    "$REF/kernels/flash_attention/10_flash_attn_v2.cu" \
    "$REF/kernels/paged_attention/11_paged_attn.cu" \
    "$REF/kernels/paged_attention/12_gqa.cu" \
    "$REF/kernels/decode/13_decode_attn.cu" \
    "$REF/kernels/quantization/14_int8_gemm.cu" \
    "$REF/kernels/layernorm/15_layernorm_residual.cu"
  # the reference's GPT2Engine (INT8 backend) with the kernels it calls; cuBLAS is linked
  # because the engine's class also holds its (unused here) cuBLAS backend
  "$NVCC" -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -shared -Xcompiler -fPIC \
    -Xcompiler -fvisibility=hidden \
    -I "$REF/include" -I "$REF/kernels" -I "$REF/src" -I "$REF" \
    -o "$HERE/_ref/libref_engine.so" \
    "$HERE/ref_engine_wrappers.cu" \
    "$REF/src/gpt2_engine.cu" \
    "$REF/src/sampler.cu" \
    "$REF/kernels/flash_attention/10_flash_attn_v2.cu" \
    "$REF/kernels/decode/13_decode_attn.cu" \
    "$REF/kernels/quantization/14_int8_gemm.cu" \
    "$REF/kernels/layernorm/15_layernorm_residual.cu" \
    "$REF/kernels/layernorm/15_embed.cu" \
    -lcublas
fi
