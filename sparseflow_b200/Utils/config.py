"""Runtime constants (reference: Utils/config.py:15-43).

PRESCAN_ACTIVITY_EPS is the prescan threshold; it is compared in IEEE half
precision, as the reference compares it against its fp16 activations.
"""
PRESCAN_ACTIVITY_EPS = 1e-6
NUMERIC_EPS = 1e-6
SPARSE_DENSE_RATIO_THRESHOLD = 0.85
# The reference ships its runtime EMA/dense-fallback policy switched off
# (Utils/config.py:43); the B200 path keeps that default and never syncs.
ENABLE_RUNTIME_FALLBACK_POLICY = False
