"""Targets: the B200 lowering of tile programs into executor launch descriptors (targets/b200)."""
