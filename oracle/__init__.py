"""CPU oracle of the Jakal-Net hot path (test infrastructure only; see oracle.oracle)."""
from .oracle import *  # noqa: F401,F403
