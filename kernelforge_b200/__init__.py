"""B200-native (sm_100a) KernelForge hot path.

Subpackages mirror the reference's operator modules and keep their call signatures:

* ``kernelforge_b200.rmsnorm``               -- one-pass RMSNorm forward
* ``kernelforge_b200.SANA_LinearAttention``  -- SANA ReLU linear attention (packed QKV)
* ``kernelforge_b200.flash_attention_jvp``   -- FlashAttention forward / forward-mode JVP

Every compute call goes through the C ABI of ``include/kernelforge_b200.h`` (library built by
``python -m kernelforge_b200.build``); importing a subpackage without the library fails.
"""

__all__ = ["rmsnorm", "SANA_LinearAttention", "flash_attention_jvp"]
