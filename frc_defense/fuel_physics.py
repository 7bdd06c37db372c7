"""`FuelPhysicsConfig` under the reference module name."""
from autodrive_b200.sim.world import FuelPhysicsConfig  # noqa: F401
