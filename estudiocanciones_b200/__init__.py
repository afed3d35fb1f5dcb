"""B200-native (sm_100a) HeartMuLa per-frame decode path for EstudioCanciones.

* :mod:`.kernels` — drop-in counterparts of the reference's ``app/kernels.py``;
* :mod:`.engine` — ``HeartMuLaLite`` with the reference engine's interface;
* :mod:`.checkpoint` — the int8 checkpoint format and synthetic weights;
* :mod:`.shard` — takes sharded over the GPUs of one box.

The compute lives in ``libheartmula_b200.so`` (C ABI: ``include/heartmula_b200.h``),
built in-tree by :mod:`.build`.
"""
__version__ = "0.1.0"
