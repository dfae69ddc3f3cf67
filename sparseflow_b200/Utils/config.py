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

# Execution-grounded dispatch thresholds (reference Utils/config.py:50-61): minimum dense MACs a
# layer's sparse path must skip per tile, by kernel family; minimum saved-work fraction; margins;
# minimum confidence for a sparse decision.
DISPATCH_TAU_3X3 = 100_000
DISPATCH_TAU_1X1 = 200_000
DISPATCH_TAU_LINEAR = 800_000
DISPATCH_TAU_ATTN_LINEAR = 900_000
DISPATCH_TAU_ATTN_MATMUL = 1_200_000
DISPATCH_R_MIN = 0.15
DISPATCH_R_MARGIN = 0.0
DISPATCH_TAU_MARGIN = 0.0
DISPATCH_MIN_CONFIDENCE = 0.60

# 3x3/s1 convolutions with at most this many input channels run on the tcgen05 implicit-GEMM kernel
# (its weight digits stay in shared memory; the library's limit for that kernel).
TC3X3_MAX_CIN = 64

# optimize(): the LIF nodes whose spikes feed a replaced convolution write those spikes' event masks
# (LIFNode.emit_event_masks), so the convolution skips its mask pass. Results are identical either
# way; SF_EMIT_EVENT_MASKS=0 in the environment turns it off.
EMIT_EVENT_MASKS = True
