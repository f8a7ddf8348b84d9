"""Analytical latency model (kvserve_v1/compression/controller/analytical_model.py).

With V the KV volume (MB), S a profile's harmonic codec speed (MB/s), B the
link bandwidth (MB/s) and cr its compression ratio:

    T_0 = T_model + V / B                       (no compression)
    T_p = T_model + V / S + V / (B * cr)        (compressed transfer)

and compression pays off (Theorem 1) iff ``B < (1 - 1/cr) * S``.

The reference's ``predict_latency`` multiplies the transfer term by cr
(``V * cr / B``, analytical_model.py:59) although its docstring and
Theorem 1 divide; ``transfer_model="reference"`` reproduces that for parity,
the default uses the corrected ``V / (B * cr)``.
"""
from __future__ import annotations

from .profile import Profile

MB = 1024.0 * 1024.0


class AnalyticalModel:
    def __init__(self, transfer_model: str = "corrected"):
        if transfer_model not in ("corrected", "reference"):
            raise ValueError("transfer_model must be 'corrected' or 'reference'")
        self.transfer_model = transfer_model

    def predict_latency(self, profile: Profile, V_bytes: float, B_mbps: float, T_model_ms: float) -> float:
        V = V_bytes / MB
        cr = profile.compression_ratio
        codec_ms = V / profile.harmonic_speed * 1e3
        if self.transfer_model == "reference":
            xfer_ms = V * cr / B_mbps * 1e3
        else:
            xfer_ms = V / (B_mbps * cr) * 1e3
        return T_model_ms + codec_ms + xfer_ms

    @staticmethod
    def predict_baseline_latency(V_bytes: float, B_mbps: float, T_model_ms: float) -> float:
        return T_model_ms + (V_bytes / MB) / B_mbps * 1e3

    @staticmethod
    def check_benefit(profile: Profile, B_mbps: float) -> bool:
        cr, S = profile.compression_ratio, profile.harmonic_speed
        return B_mbps < (1.0 - 1.0 / cr) * S

    def compute_speedup(self, profile: Profile, V_bytes: float, B_mbps: float, T_model_ms: float) -> float:
        return (self.predict_baseline_latency(V_bytes, B_mbps, T_model_ms)
                / self.predict_latency(profile, V_bytes, B_mbps, T_model_ms))
