"""B200 (sm_100a) fp16 -> fp32 GEMM and 5-D contraction: the C-ABI library in csrc/
(built to libb2g_gemm.so by build.py) and its ctypes binding b2g.py."""
