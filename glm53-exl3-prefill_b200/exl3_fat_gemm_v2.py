"""PR77 fat-GEMM drop-in on sm_100a: the functions of kernel/exl3_fat_gemm_v2.cu:328-333 and PR77's names.

    import exl3_fat_gemm_v2 as ext2
    ext2.fat_gemm_v2(a, packed, out, svh, K, mcg, mul1, variant)
    ext2.fat_gemm_v2_scatter(a, packed, out, svh, token_idx, route_weight, K, mcg, mul1, variant)
    ext2.smem_bytes(variant)
    ext2.exl3_fat_gemm(a, packed, out, svh, K, mcg, mul1)                       # PR77 name
    ext2.exl3_fat_gemm_scatter(a, packed, out, svh, tok, rw, K, mcg, mul1)     # PR77 name

All of them run the same tcgen05 trellis GEMM as the grouped path (one expert, fp32 output).
"""
import os
import sys

_HERE = os.path.dirname(os.path.abspath(__file__))
if _HERE not in sys.path:
    sys.path.insert(0, _HERE)

from b200_ext import (exl3_fat_gemm, exl3_fat_gemm_scatter, fat_gemm_v2,  # noqa: E402,F401
                      fat_gemm_v2_scatter, smem_bytes)

__all__ = ["fat_gemm_v2", "fat_gemm_v2_scatter", "smem_bytes", "exl3_fat_gemm", "exl3_fat_gemm_scatter"]
