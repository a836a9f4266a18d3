.version 8.0
.target sm_89
.address_size 64

.visible .entry k_gelu_tanh_affine(
        .param .u64 param_x,
        .param .u64 param_s,
        .param .u64 param_t,
        .param .u64 param_y
)
.reqntid 128
{
        .reg .pred      %p<2>;
        .reg .f32       %f<24>;
        .reg .b32       %r<10>;
        .reg .b64       %rd<9>;

        ld.param.u64    %rd1, [param_x];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_s];
        cvta.to.global.u64     %rd2, %rd2;
        ld.param.u64    %rd3, [param_t];
        cvta.to.global.u64     %rd3, %rd3;
        ld.param.u64    %rd4, [param_y];
        cvta.to.global.u64     %rd4, %rd4;
        mov.u32         %r1, %tid.x;
        mov.u32         %r2, %ntid.x;
        mov.u32         %r3, %ctaid.x;
        mad.lo.s32      %r4, %r3, %r2, %r1;
        mov.u32         %r5, %nctaid.x;
        shr.u32         %r6, %r4, 14;
        and.b32         %r7, %r4, 16383;
        shl.b32         %r8, %r6, 14;
        add.s32         %r9, %r8, %r7;
        mad.wide.s32    %rd5, %r9, 4, %rd1;
        ld.global.nc.f32   %f1, [%rd5];
        mad.wide.s32    %rd6, %r7, 4, %rd2;
        ld.global.nc.f32   %f2, [%rd6];
        mad.wide.s32    %rd7, %r7, 4, %rd3;
        ld.global.nc.f32   %f3, [%rd7];
        fma.rn.f32      %f4, %f1, %f2, %f3;
        mul.f32         %f5, %f4, %f4;
        mul.f32         %f6, %f5, %f4;
        mov.f32         %f7, 0f3D372713;
        fma.rn.f32      %f8, %f6, %f7, %f4;
        mov.f32         %f9, 0f3F4C422A;
        mul.f32         %f10, %f8, %f9;
        mov.f32         %f12, 0f40000000;
        mul.f32         %f13, %f10, %f12;
        mul.f32         %f15, %f13, 0f3FB8AA3B;
        ex2.approx.ftz.f32 %f14, %f15;
        mov.f32         %f16, 0f3F800000;
        sub.f32         %f17, %f14, %f16;
        add.f32         %f18, %f14, %f16;
        div.rn.f32      %f11, %f17, %f18;
        mov.f32         %f19, 0f3F800000;
        add.f32         %f20, %f11, %f19;
        mov.f32         %f21, 0f3F000000;
        mul.f32         %f22, %f4, %f21;
        mul.f32         %f23, %f22, %f20;
        mad.wide.s32    %rd8, %r9, 4, %rd4;
        st.global.f32   [%rd8], %f23;
        ret;
}
