"""The stage machine (driver/compiler.py): lower a kernel file into a kernel object, run it, verify it."""
