"""CPU restatement of voxwerk's sampler: test infrastructure only (see vw_oracle.cpp)."""
