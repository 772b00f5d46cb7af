"""CPU: the seeded acceptance scenarios reach every path of the loop body."""
from tests import accept_cases as AC


def test_scenarios_cover_every_path():
    """The seeds above reach every mode and both stop rules."""
    seen = set()
    for seed in range(24):
        for tight in (False, True):
            sc = AC.make_scenario(seed, tight=tight)
            out, _ = AC.run_oracle(sc, len(sc["blocks"]) - 1 if seed % 3 == 0 else None)
            for blk, (r, _, _) in zip(sc["blocks"], out):
                seen.add(("mode", blk["mode"]))
                seen.add(("fin", r["finished"]))
                seen.add(("unique", r["match_count"] == 1))
                seen.add(("multi", r["match_count"] > 1))
    for key in [("mode", 0), ("mode", 1), ("mode", 2), ("mode", 3), ("fin", 0), ("fin", 1),
                ("fin", 2), ("fin", 3), ("unique", True), ("multi", True)]:
        assert key in seen, key
