"""Blackwell-native FlashAttention-2 forward (drop-in for roy6n23/triton-fa2-forward's fa2)."""
