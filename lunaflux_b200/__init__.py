"""LunaFlux for NVIDIA B200: an LLM serving engine built on PyTorch and
hand-written sm_100a kernels (tcgen05 / TMEM / TMA), with tensor- and
expert-parallel serving over NVLink 5."""
__version__ = "0.1.0"
