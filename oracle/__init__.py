"""CPU oracle (test infrastructure only) — see ``tension_oracle``."""
