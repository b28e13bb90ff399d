"""CPU oracle of tpt-infer's reference kernels: test infrastructure only
(the parity checker and the timed CPU baseline), never the product path."""
