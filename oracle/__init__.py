"""ORACLE package — test infrastructure only (CPU restatement of the reference training step
and the harness that runs the reference itself). The product path never imports it."""
