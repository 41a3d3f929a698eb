"""CPU oracle and reference-path wrappers: TEST INFRASTRUCTURE ONLY."""
