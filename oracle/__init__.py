"""CPU oracle of the tinygs hot path -- test infrastructure only (see tgs_oracle.h)."""
