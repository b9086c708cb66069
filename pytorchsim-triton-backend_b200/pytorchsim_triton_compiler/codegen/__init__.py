"""B200 codegen package."""
