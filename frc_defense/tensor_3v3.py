"""`TensorThreeVsThreeEnv` under the reference module name."""
from autodrive_b200.sim.env3v3 import (  # noqa: F401
    ACTION_DIM, CONTROL_MODES, NUM_ROBOTS, OBS_DIM, TEAM_IDS, TensorThreeVsThreeEnv)
