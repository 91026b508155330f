"""CPU oracle and reference-kernel harness: test infrastructure, not product code."""
