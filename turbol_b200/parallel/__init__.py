"""turbol_b200.parallel"""
