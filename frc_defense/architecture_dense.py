"""Compatibility import path: ``frc_defense.architecture_dense`` -> ``autodrive_b200.models.zoo``."""
from autodrive_b200.models.zoo import *  # noqa: F401,F403
from autodrive_b200.models.zoo import (BaselineMLP, DeepSetsPolicy, EntityAttentionPolicy, FieldFNOPolicy,  # noqa: F401
                                      FullFieldCNN, FullFieldResNet, PerceptionActorCritic, ResidualMLP,
                                      make_policy)
