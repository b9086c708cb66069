"""What the compiler hands a device, and what a kernel file declares (the reference's contract/)."""
