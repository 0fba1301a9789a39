"""Host side of libltxattn_cuda (filled in below)."""
