"""Mesh/process groups, tensor parallelism, the ZeRO-3 engine and the NVLink transport."""
