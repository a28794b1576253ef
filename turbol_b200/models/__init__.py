"""turbol_b200.models"""
