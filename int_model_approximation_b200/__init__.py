"""B200-native student-linear hot path of int-model-approximation.

Modules mirror the reference package:
  hawkeye            <- int_model_approximation/hawkeye.py
  hawkeye_freivalds  <- int_model_approximation/hawkeye_freivalds.py
  students           <- the student side of int_model_approximation/__main__.py
plus codebook (quantiser, digit planes, tcgen05 integer GEMM), freivalds (the
product check) and synthetic (seeded workload inputs).  All compute runs in
libima_b200.so (sm_100a); see include/ima_b200.h for the C ABI.
"""

__all__ = ["codebook", "freivalds", "hawkeye", "hawkeye_freivalds", "students", "synthetic"]
