"""Drop-in replacements for the reference's `kernels/hip/*` modules.

Each module keeps the reference's public surface (`kernel_fn`, `KERNEL_TYPE`,
`BACKEND`) and calls the sm_100a kernels of libak_b200.so through
`kernels._ak`.
"""
