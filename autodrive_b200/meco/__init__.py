"""MECO research layer: candidate / goal scorers with a fail-closed arbiter,
their learning inputs, and the research operations (leases, scheduling,
supervision, attestation, release gate)."""
from .ops import (DeviceLease, MecoTaskScheduler, SupervisedTask, Supervisor, gpu_attestation,  # noqa: F401
                  native_extension_identity, release_gate)
from .tracks import (TRACKS, DecisionRequest, ScorerOutput, candidate_policy_logits, choose_candidate,  # noqa: F401
                     make_meco_track, opponent_forecast, opponent_risk_penalty)
