"""The reference arm's harness: the reference implementation installed in baseline/_ref."""
