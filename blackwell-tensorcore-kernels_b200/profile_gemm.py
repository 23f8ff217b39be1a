"""Small driver for profiling one GEMM kind under ncu: KIND=f16|fp8|fp4|mxfp4, N=size (square),
or M / N / K separately (M=128 N=65536 K=8192 is the skinny shape).
Runs the GEMM three times (ncu -s 1 -c 1 then captures the second launch). KIND=quant instead
runs three rounds of the quantisers on an N x N FP32 input: MXFP4 rows, MXFP4 columns (the Bt
operand) and a transposed E4M3 with the fixed scale (ncu -k regex:k_quant -s 3 -c 3 captures
the second round).

    KIND=f16 N=8192 ncu --set full --clock-control none -k regex:bw_tc_gemm -s 1 -c 1 \
        -o prof python blackwell-tensorcore-kernels_b200/profile_gemm.py
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import torch, bwgemm
bwgemm.init(0)
dev = torch.device('cuda:0')
kind = os.environ.get('KIND', 'f16'); n = int(os.environ.get('N', '8192'))
M = int(os.environ.get('M', n)); N = n; K = int(os.environ.get('K', n))
if kind == 'f16':
    A = torch.randn(M, K, device=dev).half(); B = torch.randn(K, N, device=dev).half(); C = torch.empty(M, N, device=dev)
    f = lambda: bwgemm.gemm_f16(A, B, C)
elif kind == 'fp8':
    qa, sa = bwgemm.quantize_fp8(torch.randn(M, K, device=dev)); qb, sb = bwgemm.quantize_fp8(torch.randn(K, N, device=dev), True)
    C = torch.empty(M, N, device=dev, dtype=torch.bfloat16); f = lambda: bwgemm.gemm_fp8(qa, qb, sa, sb, C)
elif kind == 'fp4':
    qa, sa = bwgemm.quantize_fp4(torch.randn(M, K, device=dev)); qb, sb = bwgemm.quantize_fp4(torch.randn(K, N, device=dev), True)
    C = torch.empty(M, N, device=dev, dtype=torch.bfloat16); f = lambda: bwgemm.gemm_fp4(qa, qb, K, sa, sb, C=C)
elif kind == 'quant':
    x = torch.randn(M, K, device=dev)

    def f():
        bwgemm.quantize_mxfp4(x, False)
        bwgemm.quantize_mxfp4(x, True)
        bwgemm.quantize_fp8(x, True, bwgemm.SCALE_FIXED8)
else:
    qa, sfa = bwgemm.quantize_mxfp4(torch.randn(M, K, device=dev)); qb, sfb = bwgemm.quantize_mxfp4(torch.randn(K, N, device=dev), True)
    C = torch.empty(M, N, device=dev, dtype=torch.bfloat16); f = lambda: bwgemm.gemm_mxfp4(qa, qb, sfa, sfb, K, C=C)
for _ in range(3): f()
torch.cuda.synchronize(); print('ok', bwgemm.device_status())
