"""The chunked autoregressive rollout on the B200 block."""
