"""The Craftax game as batched tensor programs: vocabularies, state, world generation, rules, observation."""
