"""B200-native SmolVLA chunk path: vision tower, prefix pass and action-expert denoising on
hand-written sm_100a CUDA, behind the so101-smolvla-edge `Engine` API."""

__version__ = "0.1.0"
