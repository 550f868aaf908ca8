"""CPU oracle package (test infrastructure only; see oracle/moe_oracle.cpp)."""
