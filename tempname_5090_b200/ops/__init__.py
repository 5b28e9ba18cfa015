"""Hand-written sm_100a operators (Python entry points over tempname_5090_b200._C)."""
