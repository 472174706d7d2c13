"""CPU oracle of the shift path — test infrastructure, never imported by ``marathon_b200``."""
