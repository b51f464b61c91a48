"""B200-native 2-D (data x tensor) parallel LLaMA training.

Sub-packages: ``config``, ``models``, ``ops`` (fused sm_100a kernels with CPU
reference paths), ``parallel`` (mesh, TP, ZeRO-3 engine, NVLink transport),
``training``, ``data``, ``checkpointing``, ``observability``, ``utils``.
"""

__version__ = "0.1.0"
