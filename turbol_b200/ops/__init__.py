"""turbol_b200.ops"""
