"""Execution devices: the CUDA launcher (cuda.py, over the native executor native.py) and the device
registry (device.py)."""
