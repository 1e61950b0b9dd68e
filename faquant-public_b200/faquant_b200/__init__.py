"""B200-native (sm_100a) HiF4 W4A4 Linear and HiF4 QK/PV attention for FAQUANT.

The Python layer mirrors the reference's operator API (``FakeQuantLinear``,
``HiF4Linear``, the ``faquant_simulated`` attention backend, Wan's
``flash_attention`` drop-in) and calls the C-ABI library
``libfaquant_b200.so`` built from ``csrc/``. There is no CPU fallback: every
operator raises if the library or a CUDA device is missing.
"""

__version__ = "0.1.0"
