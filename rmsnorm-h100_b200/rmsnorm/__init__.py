# SPDX-License-Identifier: MIT
"""rmsnorm -- drop-in replacement for the `rmsnorm` package of Int21-AI/RMSNorm-H100,
computing on NVIDIA B200 (sm_100a) through librmsnorm_b200 (C ABI: include/rmsnorm_b200.h).

Exports the reference's public names (rmsnorm/__init__.py:4-32 of the reference)."""

from .rmsnorm import (
    QuackRMSNorm,
    RMSNormFunction,
    layernorm_fwd,
    layernorm_mean_ref,
    layernorm_ref,
    layernorm_rstd_ref,
    rmsnorm,
    rmsnorm_bwd,
    rmsnorm_bwd_ref,
    rmsnorm_bwd_tuned,
    rmsnorm_fwd,
    rmsnorm_fwd_tuned,
    rmsnorm_ref,
)

__all__ = [
    "QuackRMSNorm",
    "layernorm_fwd",
    "layernorm_mean_ref",
    "layernorm_ref",
    "layernorm_rstd_ref",
    "rmsnorm",
    "rmsnorm_bwd",
    "rmsnorm_bwd_ref",
    "rmsnorm_bwd_tuned",
    "rmsnorm_fwd",
    "rmsnorm_fwd_tuned",
    "rmsnorm_ref",
]
