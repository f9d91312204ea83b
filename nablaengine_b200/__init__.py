"""nablaengine_b200: a B200-native (sm_100a) batched physics step for the mjlab Unitree G1, behind the API of
OamIcs/NablaEngine's `torch_ffi` (step / forward) and a C ABI (include/nabla_g1.h, libnabla_g1.so)."""
__version__ = "0.1.0"
