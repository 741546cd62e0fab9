"""CPU oracle package (test infrastructure only; see vox_oracle.h)."""
