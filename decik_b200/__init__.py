"""decik_b200: a B200-native (sm_100a) rebuild of the attention block of decik's NF4 QLoRA step.

- ``decik_b200.ops``       torch-tensor front end of the C ABI (``include/decik_b200.h``)
- ``decik_b200.solution``  the reference-facing patch surface (``solution.apply()`` and the
                           autograd Functions of solution/nf4.py, attn.py, varlen.py, rmsnorm.py)
- ``decik_b200.build``     builds ``decik_b200/lib/libdecik_b200.so`` with nvcc for sm_100a
"""

__all__ = ["ops", "solution"]
