#!/usr/bin/env bash
# Compiles the reference's own GEMM launchers (waynehacking8/blackwell-tensorcore-kernels,
# src/*.cu) for sm_100a from the sources where they lie, plus oracle/ref_shim.cu, into
# oracle/_ref/libref_kernels.so. Nothing is copied into this repository; the output is
# git-ignored and travels to the GPU box with the checkout.
# Built: wmma, mma_* (mma.sync), mma_fp8, cublas, cublas_tc, cublas_tf32, cublaslt_fp8.
# Not built: cutlass_sm90.cu (sm_90a wgmma only), the FP4/MXFP4 paths (sm_120a-only PTX,
# guarded by BUILD_SM120A), mma_rate_probe.cu (its own binary).
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
# The reference checkout: BW_REFERENCE_DIR, else a directory named "reference" beside this
# repository's own directory.
REF=${BW_REFERENCE_DIR:-$HERE/../../reference}
OUT="$HERE/_ref"
[ -d "$REF/src" ] || { echo "reference sources not found at $REF" >&2; exit 1; }
mkdir -p "$OUT/obj"
SRCS="gemm_naive gemm_tiled gemm_wmma gemm_mma gemm_mma_fp8 reference cublas_tc cublas_tf32 cublaslt_fp8"
STAMP="$OUT/libref_kernels.so"
need=0
[ -f "$STAMP" ] || need=1
for s in $SRCS; do [ "$REF/src/$s.cu" -nt "$STAMP" ] && need=1; done
[ "$HERE/ref_shim.cu" -nt "$STAMP" ] && need=1
[ $need -eq 0 ] && exit 0
NV="nvcc -std=c++17 -O3 -gencode arch=compute_100a,code=sm_100a -Xcompiler -fPIC -I$REF/include"
for s in $SRCS; do $NV -c "$REF/src/$s.cu" -o "$OUT/obj/$s.o"; done
$NV -c "$HERE/ref_shim.cu" -o "$OUT/obj/ref_shim.o"
nvcc -gencode arch=compute_100a,code=sm_100a -shared -o "$STAMP" "$OUT"/obj/*.o -lcublas -lcublasLt
echo "built $STAMP"
