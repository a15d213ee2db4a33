"""TEST INFRASTRUCTURE ONLY: the CPU restatement of the tcgen05_model
arithmetic used as the parity reference.  Not part of the product path."""
