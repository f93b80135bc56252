"""CPU oracle for the quantized-inference hot path -- test infrastructure only."""
