"""turbol_b200.rl"""
