"""vdttfs -- Python mirror of the B200 VD-TTFS engine's C ABI (include/vdttfs.h).

The engine itself is C++/CUDA in ``libvdttfs.so`` (vd-ttfs_b200/csrc); this
package holds the network descriptors, the weight-blob format, the seeded
synthetic workloads and a ctypes binding whose names follow the reference's
host helpers (update_LUTs, k_bucketize, k_conv_bucketed, ...).
"""
from . import blob, nets, synth  # noqa: F401

__all__ = ["blob", "nets", "synth"]
