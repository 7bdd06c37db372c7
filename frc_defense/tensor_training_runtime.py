"""Model/runtime helpers under the reference module name."""
from autodrive_b200.models.actor_critic import (  # noqa: F401
    ACTION_DIM, OBS_DIM, STRATEGIC_ACTION_DIM, ActorCritic, DDPScore as _DDPScore)
from autodrive_b200.parallel.dist import distributed_state as _distributed_state  # noqa: F401
from autodrive_b200.train.ppo import (  # noqa: F401
    CURRICULUM_STAGES, DEFENSE_TRAINING_OPPONENTS, OBS_NORMALIZATION, STATIC_OPPONENT_FRACTION,
    curriculum_opponents as _curriculum_opponents, curriculum_stage as _curriculum_stage)
from autodrive_b200.train.rollout import gae_advantages as _gae_advantages  # noqa: F401
