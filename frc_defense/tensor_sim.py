"""`TensorDefenseEnv` under the reference module name."""
from autodrive_b200.sim.env_defense import TensorDefenseEnv  # noqa: F401
from autodrive_b200.sim.world import SwerveParameters as TensorSwerveParameters  # noqa: F401
