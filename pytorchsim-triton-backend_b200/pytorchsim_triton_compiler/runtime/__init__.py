"""B200 runtime package."""
