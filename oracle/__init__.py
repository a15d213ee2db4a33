"""TEST INFRASTRUCTURE ONLY: the CPU restatement of the tcgen05_model
arithmetic used as the parity checker.  Not part of the product path."""
