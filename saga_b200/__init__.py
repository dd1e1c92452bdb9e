"""saga_b200: SAGA's decode-time Atop-N attention on NVIDIA B200 (sm_100a).

Layers:
  include/saga_b200.h        C ABI (libsaga_b200.so, built from saga_b200/csrc)
  saga_b200._lib             ctypes binding of that ABI
  saga_b200.ops              torch-facing host layer + torch.ops.saga custom ops
  saga_b200.attention        drop-in for the reference's attention/ package
  saga_b200.workloads        seeded synthetic decode inputs
"""
__version__ = "0.1.0"
