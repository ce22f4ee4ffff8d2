"""mace_onegpu (B200 build): the exact receiver-chunked three-pass MACE force evaluation on sm_100a.

Module paths mirror the reference package (ShiQiaoL/mace-million) for the drop-in surface:
``mace_onegpu.mliap_threepass.ThreePassMLIAP`` (LAMMPS ML-IAP plugin) and ``mace_onegpu.fused_conv.FusedConvTP``.
The arithmetic runs in libmace_b200.so (csrc/, C ABI in include/mace_b200.h); this package is the host side.
"""
__version__ = "0.1.0+b200"
