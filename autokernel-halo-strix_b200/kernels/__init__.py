"""B200 (sm_100a) kernels behind the autokernel drop-in API.

Module paths mirror the reference project (`kernels.hip.*`, `kernels.ce_fused`)
so that code written against it imports these modules unchanged.  The
`hip` sub-package name is kept only for import compatibility: every kernel in
it is a CUDA kernel in libak_b200.so.
"""
