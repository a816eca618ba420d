"""CPU oracle package — test infrastructure only (see myos_oracle.h)."""
