"""placemoe_b200: a Blackwell-native MoE training framework with profile-guided expert placement."""

__version__ = "0.1.0"
