"""Host side of the sm_100a VC-Attention kernels (libvcattn.so)."""
