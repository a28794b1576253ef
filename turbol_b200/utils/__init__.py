"""turbol_b200.utils"""
