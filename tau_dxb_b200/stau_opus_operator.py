"""Reference-named module: the drop-in for echo/stau_opus_operator.py.

Exports the names the reference's callers import from that module
(STauOpusAttentionFunction, STauOpusAttentionModule, CLAMP_MIN,
_log_tau_for_init, init_log_tau_from_values), backed by the B200 kernels.
"""
from .attention import (CLAMP_MIN, STauOpusAttentionFunction,  # noqa: F401
                        STauOpusAttentionModule, _log_tau_for_init,
                        init_log_tau_from_values)
