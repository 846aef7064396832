"""B200-native MoE expert-FFN hot path (host-side Python mirror).

Import name: ``moe_b200`` (the directory name is not a Python identifier;
tests/conftest.py and bench.py register it under that name).
"""
