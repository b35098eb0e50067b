"""Hardware probes behind the design of the flash-attention kernels (not used by the library)."""
