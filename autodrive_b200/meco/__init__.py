"""MECO research layer: candidate / goal scorers with a fail-closed arbiter,
their learning inputs, training and evaluation on the offense curriculum, the
production adapter, and the research operations (leases, scheduling,
supervision, attestation, release gate)."""
from .adapter import (DiagnosticMonitor, MecoInferenceRequest, ProductionMecoAdapter, capture_request,  # noqa: F401
                      export_scorer, profile_latency)
from .ops import (DeviceLease, MecoTaskScheduler, SupervisedTask, Supervisor, gpu_attestation,  # noqa: F401
                  native_extension_identity, release_gate)
from .tracks import (TRACKS, DecisionRequest, ScorerOutput, candidate_policy_logits, choose_candidate,  # noqa: F401
                     make_meco_track, opponent_forecast, opponent_risk_penalty)
from .train import (MecoConfig, MecoPolicy, MetricLedger, counterfactual_labels, evaluate_meco,  # noqa: F401
                    supervised_warm_start, train_meco)
