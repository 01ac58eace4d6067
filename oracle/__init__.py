"""CPU oracle of the batch-invariant kernels -- test infrastructure only."""
