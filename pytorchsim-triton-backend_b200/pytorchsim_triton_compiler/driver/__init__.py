"""B200 driver package."""
