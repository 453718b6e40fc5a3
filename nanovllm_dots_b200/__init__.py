"""B200-native MeanFlow FM head for dots.tts (sm_100a CUDA behind a C ABI)."""
__all__ = ["synthetic"]
