"""B200 targets/b200 package."""
