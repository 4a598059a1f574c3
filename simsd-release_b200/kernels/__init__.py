"""B200 (sm_100a) drop-in for SimSD's `kernels` package: thin-M linear and fused MoE dispatch.

Put `simsd-release_b200/` ahead of the reference checkout on `sys.path` and
`from kernels import fused_toggle` resolves here; the operator signatures are
the reference's (kernels/fused_toggle.py, kernels/thin_linear_fused.py,
kernels/moe_dispatch_fused.py).  The compute lives in libsimsd_b200.so.
"""
