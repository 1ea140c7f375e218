"""Minimal MLX-API shim used ONLY by tests/golden/gen_golden.py.

It lets the reference's unmodified ``mirror_sd/dflash.py`` and the quantiser
in ``mirror_sd/ane_model.py`` run in this container (MLX is not installable
here) so their composition can be frozen as golden fixtures.  Arrays are
numpy arrays; every op is a restatement of the documented MLX semantics.
"""
