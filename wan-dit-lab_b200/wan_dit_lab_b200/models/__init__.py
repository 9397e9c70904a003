"""The Wan block on the B200 operators."""
