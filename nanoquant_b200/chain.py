"""Input modes of the grouped decode GEMV (``nq_gemv_group_ex`` / ``nq_gemv_group_tp``,
include/nq_b200.h ``NQ_CHAIN_X_*``): the layers of a launch read x' formed in the kernel's
prologue from its neighbours' outputs -- x' = x (PLAIN), RMSNorm(x + residual) * weight
(RMSNORM), silu(x) * x2 (SILU_MUL) or x * x2 (MUL).  The reference runs these neighbours as HF
modules between its per-linear kernel calls (src/nanoquant/modules/linear.py:155-164)."""

PLAIN, RMSNORM, SILU_MUL, MUL = 0, 1, 2, 3
