"""CPU oracle for the mHC operators (test infrastructure only; see mhc_oracle)."""
