"""face_b200: B200-native (sm_100a) engine for face-mlip's energy+force evaluation hot path.

Modules mirror the reference package `face`:
  model        FACE (face/model.py)            kernels     factor_density (face/kernels.py)
  node_kernel  node_algebra (face/node_kernel.py)   neighbors   padded_graph (face/neighbors.py)
  electrostatics  PME / Ewald pieces (face/electrostatics.py)   calculator  load_face, FACECalculator
The native library libfacek.so (C ABI, include/facek.h) is loaded on first use.
"""
__version__ = "0.1.0"
