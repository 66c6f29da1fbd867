"""CPU oracle (test infrastructure only: used by tests/, smoke() and the CPU baseline)."""
