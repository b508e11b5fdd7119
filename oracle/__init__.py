"""CPU oracle of the higgs decode hot path -- test infrastructure only (never imported by higgs_b200)."""
