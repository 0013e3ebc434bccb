"""CPU oracle (test infrastructure only): a numpy restatement of the reference
hot/cold decode path, pinned by the golden vectors under tests/golden/."""
