"""The Triton backend plugin's Python side, B200 edition: the launcher registry (driver.set_launcher) that a
device owner hooks, kept call-compatible with the reference's pytorchsim_triton_backend package."""
