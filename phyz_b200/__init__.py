"""phyz_b200 — a B200-native batched rigid-body stepper with phyz-gpu's
batched-simulation API (BatchSim) over the C ABI of libphyzb200.so."""
from ._lib import PhyzbError
from .batch_sim import BatchSim, BodyContactGains, BodyPlane, PdDof
from .policy import ObsOp, PolicySpec
from .model import Geometry, Heightfield, Joint, Model, ModelBuilder, SpatialInertia, Transform

__all__ = ["BatchSim", "BodyContactGains", "BodyPlane", "PdDof", "PhyzbError", "ObsOp", "PolicySpec", "Geometry", "Heightfield", "Joint", "Model",
           "ModelBuilder", "SpatialInertia", "Transform"]
